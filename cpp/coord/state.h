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

// How spares may stand (policy "spares"): a spare on a device of another class than its
// position's is admitted only when `allow_mismatched` and its slowdown is within
// `max_degrade_percent` (0: any).
struct SparePoolPolicy {
  uint32_t per_engine = 0;
  int32_t loading = 0;  // policy.v1.SparePool.Loading
  bool allow_mismatched = false;
  uint32_t max_degrade_percent = 0;
};

struct Policy {
  std::vector<int32_t> outcomes;  // signals::Outcome values, in preference order
  uint32_t max_concurrent_losses = 0;  // 0: no limit
  uint32_t notice_min_ms = 0;
  bool cover_enabled = false;       // plan groups ahead of losses (policy "cover.enabled")
  uint32_t cover_max_groups_per_gpu = 0;
  SparePoolPolicy spares;
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
  std::string pool;         // the pool it was launched for ("" an engine's own spare)
};

// A pool of spare capacity for engines of one shape (spec.v1.PoolSpec as proto3 JSON): how many
// spares it wants standing, on which device class and in which domain, and how a daemon starts
// one (`{pool}`, `{device}`, `{node}`, `{socket}`, `{engines}` filled in).
struct PoolSpec {
  std::string name;
  std::vector<std::string> engines;
  uint32_t wants = 0;
  std::string device_class, domain, reason;
  std::vector<std::string> command;
  std::map<std::string, std::string> env;
  uint64_t generation = 0;
};
bool parse_pool(const std::string& json, PoolSpec& out, std::string& err);
std::string pool_json(const PoolSpec& p);

// Where a pool's next launches go: free devices (no worker, spare or launch on them) of linked,
// uncordoned nodes, of the pool's class (a substring of the product name, "" any) and domain
// ("" any), spread over nodes (one per node per round, nodes in name order), at most `count`.
struct FreeDevice {
  std::string node;
  uint32_t device = 0;
  std::string cls, domain;
};
std::vector<std::pair<std::string, uint32_t>> place_pool_spares(const PoolSpec& pool,
                                                                 const std::vector<FreeDevice>& free, uint32_t count);

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
