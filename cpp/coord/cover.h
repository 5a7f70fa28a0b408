// The cover planner: which communicator groups an engine forms ahead of a loss (pure function).
//
// A membership change is fast only if the groups of the new member set already exist. For each
// standing spare the plan names the replacement set (the current ranks with the spare in the
// position it stands for; an any-rank spare covers every position, budget permitting) and the
// current set itself, and for each set the groups that have to be formed by the processes:
// one pipeline group per tensor column (fabric scope) when the engine is pipeline-parallel.
// Tensor-parallel groups are member tables over peer memory and need no formation, so they are
// not planned. Groups shared by several sets are planned once. A per-GPU budget caps how many
// planned groups a process may hold; sets beyond it are left uncovered.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "everserve_pb.h"
#include "state.h"

namespace es {

struct CoverInput {
  std::string engine;
  uint64_t epoch = 0;
  uint32_t tp = 1, pp = 1;
  std::map<uint32_t, std::pair<std::string, uint32_t>> holders;  // rank -> (node, device)
  std::vector<SpareSeat> spares;
  uint32_t max_groups_per_gpu = 0;  // 0: no cap
};

// The plan (generation left 0: the caller numbers plans) and, per set, the ranks it covers.
signals::CoverPlan plan_cover(const CoverInput& in, std::vector<std::vector<uint32_t>>* covers = nullptr);

// A canonical text key of a group's spans ("0,R1@n0:2,2"), for matching reports to groups.
std::string spans_key(const std::vector<signals::SetMember>& spans);

}  // namespace es
