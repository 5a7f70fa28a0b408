// The coordinator's policy view and outcome choice (pure functions, no I/O).
#pragma once

#include <cstdint>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "util.h"

namespace es {

struct SpareSlotPolicy {
  std::string node;
  uint32_t device = 0;
  int64_t rank = -1;  // -1: any rank
};

struct EnginePolicy {
  std::string name;
  uint32_t tensor = 1, pipeline = 1, data = 1, expert = 1;
  bool placement_independent = false;
  std::vector<std::string> spare_nodes;
  int64_t release_bound_ms = -1;
  std::vector<std::string> replica_nodes;     // whose stores take the ranks' rows (empty: the spares' nodes)
  std::vector<SpareSlotPolicy> spare_slots;   // where the daemons launch this engine's spares
  std::vector<std::string> launch_command;    // how (empty: the engine launches its own)
  std::map<std::string, std::string> launch_env;
};

struct Policy {
  std::vector<int32_t> outcomes;  // signals::Outcome values, in preference order
  uint32_t max_concurrent_losses = 0;  // 0: no limit
  uint32_t notice_min_ms = 0;
  bool cover_enabled = false;       // plan groups ahead of losses (policy "cover.enabled")
  uint32_t cover_max_groups_per_gpu = 0;
  std::map<std::string, EnginePolicy> engines;
  uint32_t world_size(const std::string& engine) const;
};

// proto3 JSON of everserve.policy.v1.Policy (the fields the coordinator uses).
bool parse_policy(const std::string& json, Policy& out, std::string& err);

struct SpareSeat {
  std::string node;
  uint32_t device = 0;
  int64_t for_rank = -1;  // -1: any rank
  uint32_t pid = 0;
  std::string fingerprint;  // what must match the engine's ranks for an exact take ("" unknown)
};

struct Choice {
  int32_t outcome = 0;  // 0: none possible (abandon)
  std::vector<std::pair<uint32_t, SpareSeat>> take;  // lost rank -> spare that takes it
  std::string why;
};

// REPLACE when a spare stands for every lost rank (its own rank first, then any-rank spares in
// node order), else SHRINK when the policy allows it and the model is placement independent,
// else nothing: the engine is abandoned. The preference order is the policy's.
// A spare whose fingerprint is known and differs from the engine's (another build, model, KV
// format or step configuration) is not eligible.
Choice choose_outcome(const Policy& p, const std::string& engine, const std::set<uint32_t>& lost,
                      const std::vector<SpareSeat>& spares, const std::string& fingerprint = "");

}  // namespace es
