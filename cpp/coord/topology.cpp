#include "topology.h"

#include <algorithm>
#include <cctype>
#include <cmath>
#include <cstdio>

namespace es {

double class_bandwidth(const std::string& cls) {
  std::string c;
  for (char ch : cls) c.push_back((char)std::toupper((unsigned char)ch));
  // most specific names first: "GB200" before "B200", "H100 PCIE" before "H100"
  static const std::pair<const char*, double> kTable[] = {
      {"GB300", 8.0}, {"B300", 8.0}, {"GB200", 8.0}, {"B200", 8.0}, {"B100", 8.0},
      {"GH200", 4.9}, {"H200", 4.8}, {"H20", 4.0},   {"H100 NVL", 3.9}, {"H100 PCIE", 2.0},
      {"H100", 3.35}, {"H800", 3.35}, {"A100-SXM4-40GB", 1.55}, {"A100-PCIE-40GB", 1.55},
      {"A100", 2.0},  {"A800", 2.0}, {"MI300X", 5.3}, {"L40S", 0.864}, {"L40", 0.864},
      {"A40", 0.696}, {"A10", 0.6},  {"L4", 0.3},    {"T4", 0.32}};
  for (auto& [name, bw] : kTable)
    if (c.find(name) != std::string::npos) return bw;
  return 0.0;
}

static std::string gib(uint64_t b) {
  char buf[32];
  std::snprintf(buf, sizeof buf, "%.1f GiB", (double)b / (1ull << 30));
  return buf;
}

Fit fit(const Position& p, const Device& d) {
  Fit f;
  const std::string dom = d.domain.empty() ? d.node : d.domain;
  f.same_domain = p.domain.empty() || p.domain == dom;
  f.same_class = p.cls.empty() || p.cls == d.cls;
  if (p.memory_bytes > 0 && d.memory_bytes < p.memory_bytes) {
    f.why = d.cls + " has " + gib(d.memory_bytes) + ", the position needs " + gib(p.memory_bytes);
    return f;
  }
  f.ok = true;
  if (f.same_class) {
    f.speed = 1.0;
    return f;
  }
  const double from = class_bandwidth(p.cls), to = class_bandwidth(d.cls);
  if (from > 0 && to > 0) {
    f.speed = to / from;
    f.why = d.cls + " in place of " + p.cls;
  } else {
    f.speed = std::nan("");
    f.why = d.cls + " in place of " + p.cls + ": relative speed unknown";
  }
  return f;
}

bool within_degrade(const Fit& f, uint32_t max_degrade_percent) {
  if (!f.ok) return false;
  if (std::isnan(f.speed)) return max_degrade_percent == 0;
  if (max_degrade_percent == 0) return true;
  const double slowdown = (1.0 - std::min(1.0, f.speed)) * 100.0;
  return slowdown <= (double)max_degrade_percent + 1e-9;
}

void Topology::set_node(const std::string& node, std::vector<Device> devices) {
  for (auto& d : devices) {
    d.node = node;
    if (d.domain.empty()) d.domain = node;
  }
  devices_[node] = std::move(devices);
}

const Device* Topology::device(const std::string& node, uint32_t index) const {
  auto it = devices_.find(node);
  if (it == devices_.end()) return nullptr;
  for (auto& d : it->second)
    if (d.index == index) return &d;
  return nullptr;
}

const std::vector<Device>* Topology::node(const std::string& node) const {
  auto it = devices_.find(node);
  return it == devices_.end() ? nullptr : &it->second;
}

std::string Topology::domain_of(const std::string& node) const {
  auto it = devices_.find(node);
  if (it == devices_.end() || it->second.empty()) return node;
  return it->second.front().domain;
}

}  // namespace es
