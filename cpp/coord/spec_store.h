// The coordinator's spec store: what must outlive a coordinator (its standby, or its restart,
// reads it back). Keys and what they hold:
//   <engine>.status       spec.v1.EngineStatus: assignments and the change log (written BEFORE a
//                         change is delivered, so a new holder finishes a change it did not start)
//   pools/<name>.json     a pool's spec (spec.v1.PoolSpec as proto3 JSON) with its generation
//   nodes/<name>.json     a node's spec (cordoned, drain deadline, reason)
//
//   --spec-store DIR        files under DIR, each replaced atomically (rename over)
//   --spec-store k8s:NS     EverserveState custom resources (everserve.ai/v1) in namespace NS,
//                           one per key: spec.key and spec.data (base64); a write replaces the
//                           object at the resourceVersion read (the CRD is in the Helm chart)
//
// Reference parity: controller/src/spec/{mod,kubernetes}.rs (file and EverserveState backends
// of the same desired state and change log).
#pragma once

#include <map>
#include <memory>
#include <string>

#include "kube.h"

namespace es {

class SpecStore {
 public:
  virtual ~SpecStore() = default;
  virtual bool put(const std::string& key, const std::string& bytes) = 0;
  virtual bool remove(const std::string& key) = 0;
  // Every key under `prefix` ("" every key), with its bytes.
  virtual bool list(const std::string& prefix, std::map<std::string, std::string>& out) = 0;
  virtual std::string where() const = 0;
};

// nullptr for "" (no spec store).
std::unique_ptr<SpecStore> make_spec_store(const std::string& spec);

// A key as a Kubernetes object name: lower case, [a-z0-9-], a digest suffix keeping keys apart.
std::string object_name_of(const std::string& key);

}  // namespace es
