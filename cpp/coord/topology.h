// Devices, the positions engines need, and the fit between them (pure functions, no I/O).
//
// A daemon reports its node's GPUs in its hello (index, driver UUID, product name as the class,
// memory, and the domain it reaches at full speed: the node unless the daemon is told a wider
// NVLink domain). A position is one rank of one engine: the class of the device it runs on and
// what it needs. `fit` is the one place classes are compared: memory decides whether a device can
// hold a position, the class ratio estimates its speed there, and the domain is reported for the
// policy to weigh.
//
// Reference parity: controller/src/topology/mod.rs:17-225 (Device, Position, Fit, fit,
// within_degrade, Topology). The speed estimate here is this file's own: decode is bound by
// memory bandwidth, so a class's speed is its published HBM bandwidth.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace es {

struct Device {
  std::string node;
  uint32_t index = 0;
  std::string uuid;
  std::string cls;  // the product name the driver reports
  uint64_t memory_bytes = 0;
  std::string domain;  // "" is read as the node
};

struct Position {
  std::string engine;
  uint32_t rank = 0;
  uint64_t memory_bytes = 0;  // 0: unknown
  std::string cls;            // "" unknown
  std::string domain;         // "" unknown
};

struct Fit {
  bool ok = false;
  bool same_class = false;
  double speed = 0.0;  // relative to the position's class; NaN when a class has no known figure
  bool same_domain = false;
  std::string why;
};

// Published HBM bandwidth of a device class in TB/s, 0 when unknown.
double class_bandwidth(const std::string& cls);

Fit fit(const Position& p, const Device& d);

// Whether `f`'s slowdown is within `max_degrade_percent` (0: any known slowdown; an unknown speed
// passes only then).
bool within_degrade(const Fit& f, uint32_t max_degrade_percent);

class Topology {
 public:
  void set_node(const std::string& node, std::vector<Device> devices);
  void remove_node(const std::string& node) { devices_.erase(node); }
  const Device* device(const std::string& node, uint32_t index) const;
  const std::vector<Device>* node(const std::string& node) const;
  std::string domain_of(const std::string& node) const;
  const std::map<std::string, std::vector<Device>>& all() const { return devices_; }

 private:
  std::map<std::string, std::vector<Device>> devices_;
};

}  // namespace es
