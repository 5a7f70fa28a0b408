// The cover planner: which member sets an engine forms groups for ahead of a loss (pure function).
//
// A membership change is fast only if the groups of the new member set already exist. The plan
// names, within a budget of planned groups per GPU and in this order:
//   1. the current set (always: its groups are the ones serving);
//   2. for each loss the placement can suffer, node losses first (every rank a node holds), then
//      single positions on nodes that hold more than one: the REPLACE set (each lost position held
//      by its own standing spare, else by the any-rank spare holding the fewest planned groups so
//      far, never a spare on a node the loss takes whole) and, when the policy allows SHRINK, the
//      survivors' set;
//   3. for each single-position loss already covered, a second spare's REPLACE set (a spare other
//      than those in the sets that cover it), so a second failure of that position is covered too.
// Losses no set answers are reported with the reason (over the budget, no spare can take them, or
// the policy allows neither outcome).
//
// Groups: a tensor-parallel group is a member table over peer memory and needs no formation, so
// only pipeline groups are planned: one per tensor column spanning the set's members of that
// column in stage order, when the engine has stages to link. A group that several sets need is
// planned once and counted once against each process it spans (a spare counted once whatever
// position it stands for).
//
// Reference parity: controller/src/policy/cover.rs:1-12,277-386 (the same order of sets, the
// budget rule and the uncovered reasons; this planner's own structure and data types).
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
  std::vector<SpareSeat> spares;                                 // in pool order
  uint32_t max_groups_per_gpu = 0;                               // 0: no cap
  bool replace = true;                                           // the policy allows REPLACE
  bool shrink = false;                                           // ... and SHRINK
  // groups other engines' plans already put on a spare ((node, device) -> count): a pool's spare
  // stands for several engines at once, and the budget counts across them
  std::map<std::pair<std::string, uint32_t>, uint32_t> elsewhere;
};

struct Uncovered {
  std::vector<uint32_t> lost;
  std::string why;
};

// The plan (generation left 0: the caller numbers plans), per set the ranks whose loss it
// answers, and the losses no set answers.
signals::CoverPlan plan_cover(const CoverInput& in, std::vector<std::vector<uint32_t>>* covers = nullptr,
                              std::vector<Uncovered>* uncovered = nullptr);

// The losses a placement can suffer that the plan answers, in order: each node's ranks, then each
// position on a node that holds more than one.
std::vector<std::vector<uint32_t>> losses_of(const std::map<uint32_t, std::pair<std::string, uint32_t>>& holders);

// Whether `members` is a set the engine moves to on losing `lost`: no lost rank serves in it, every
// other position is its serving rank, and the lost positions are all held by spares or all gone.
bool answers(const std::vector<signals::SetMember>& members, const std::vector<uint32_t>& lost);

// A canonical text key of a group's spans ("0,R1@n0:2,2"), for matching reports to groups.
std::string spans_key(const std::vector<signals::SetMember>& spans);

}  // namespace es
