#include "cover.h"

#include <algorithm>

namespace es {

static signals::SetMember rank_member(uint32_t r) {
  signals::SetMember m;
  m.has_rank = true;
  m.rank = r;
  return m;
}

static signals::SetMember spare_member(uint32_t for_rank, const SpareSeat& s) {
  signals::SetMember m;
  m.has_spare = true;
  m.spare.for_rank = for_rank;
  m.spare.node = s.node;
  m.spare.device = s.device;
  return m;
}

std::string spans_key(const std::vector<signals::SetMember>& spans) {
  std::string k;
  for (size_t i = 0; i < spans.size(); i++) {
    if (i) k += ",";
    const auto& m = spans[i];
    if (m.has_spare)
      k += "R" + std::to_string(m.spare.for_rank) + "@" + m.spare.node + ":" + std::to_string(m.spare.device);
    else
      k += std::to_string(m.rank);
  }
  return k;
}

static std::string holder_of(const signals::SetMember& m, const CoverInput& in) {
  if (m.has_spare) return m.spare.node + ":" + std::to_string(m.spare.device);
  auto it = in.holders.find(m.rank);
  return it == in.holders.end() ? "?" : it->second.first + ":" + std::to_string(it->second.second);
}

signals::CoverPlan plan_cover(const CoverInput& in, std::vector<std::vector<uint32_t>>* covers) {
  signals::CoverPlan plan;
  plan.engine = in.engine;
  plan.epoch = in.epoch;
  const uint32_t world = in.tp * in.pp;
  for (auto& [r, h] : in.holders) {
    signals::Holder ho;
    ho.node = h.first;
    ho.device = h.second;
    plan.placement[r] = ho;
  }
  // candidate sets: the current one, then one replacement set per (spare, position it can take)
  struct Cand {
    std::vector<signals::SetMember> members;
    std::string purpose;
    std::vector<uint32_t> covers;
  };
  std::vector<Cand> cands;
  {
    Cand cur;
    for (uint32_t r = 0; r < world; r++) cur.members.push_back(rank_member(r));
    cur.purpose = "current";
    cands.push_back(cur);
  }
  std::vector<bool> taken(world, false);
  for (const auto& s : in.spares) {
    std::vector<uint32_t> positions;
    if (s.for_rank >= 0 && (uint32_t)s.for_rank < world)
      positions.push_back((uint32_t)s.for_rank);
    else if (s.for_rank < 0)
      for (uint32_t r = 0; r < world; r++) positions.push_back(r);
    for (uint32_t r : positions) {
      Cand c;
      for (uint32_t q = 0; q < world; q++) c.members.push_back(q == r ? spare_member(r, s) : rank_member(q));
      c.purpose = "replace rank " + std::to_string(r) + " by " + s.node + ":" + std::to_string(s.device);
      c.covers.push_back(r);
      cands.push_back(c);
    }
  }
  // groups per set: one pipeline group per column (stage order) when there are stages to link
  std::map<std::string, uint32_t> group_index;
  std::map<std::string, uint32_t> per_holder;
  for (auto& c : cands) {
    std::vector<std::vector<signals::SetMember>> groups;
    if (in.pp > 1) {
      for (uint32_t col = 0; col < in.tp; col++) {
        std::vector<signals::SetMember> spans;
        for (uint32_t st = 0; st < in.pp; st++) spans.push_back(c.members[st * in.tp + col]);
        groups.push_back(spans);
      }
    }
    // the budget: count the new groups each holder would join
    std::map<std::string, uint32_t> add;
    for (auto& g : groups)
      if (!group_index.count(spans_key(g)))
        for (auto& m : g) add[holder_of(m, in)]++;
    bool fits = true;
    if (in.max_groups_per_gpu)
      for (auto& [h, n] : add)
        if (per_holder[h] + n > in.max_groups_per_gpu) fits = false;
    if (!fits) continue;
    for (auto& [h, n] : add) per_holder[h] += n;
    signals::CoverSet set;
    set.members = c.members;
    set.purpose = c.purpose;
    for (auto& g : groups) {
      const std::string k = spans_key(g);
      auto it = group_index.find(k);
      if (it == group_index.end()) {
        signals::CoverGroup cg;
        cg.scope = signals::Scope_SCOPE_FABRIC;
        cg.spans = g;
        cg.server = g.front();
        cg.has_server = true;
        it = group_index.emplace(k, (uint32_t)plan.groups.size()).first;
        plan.groups.push_back(cg);
      }
      set.groups.push_back(it->second);
    }
    plan.sets.push_back(set);
    if (covers) covers->push_back(c.covers);
  }
  return plan;
}

}  // namespace es
