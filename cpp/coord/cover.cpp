#include "cover.h"

#include <algorithm>
#include <set>

namespace es {

namespace {

signals::SetMember rank_member(uint32_t r) {
  signals::SetMember m;
  m.has_rank = true;
  m.rank = r;
  return m;
}

signals::SetMember spare_member(uint32_t for_rank, const SpareSeat& s) {
  signals::SetMember m;
  m.has_spare = true;
  m.spare.for_rank = for_rank;
  m.spare.node = s.node;
  m.spare.device = s.device;
  return m;
}

uint32_t position_of(const signals::SetMember& m) { return m.has_spare ? m.spare.for_rank : m.rank; }

// The process a member is, for the budget: a rank by its number, a spare by its seat.
std::string process_of(const signals::SetMember& m) {
  return m.has_spare ? "S" + m.spare.node + ":" + std::to_string(m.spare.device) : "R" + std::to_string(m.rank);
}

using Seat = std::pair<std::string, uint32_t>;

// The plan being built, with what each process holds so far.
struct Builder {
  const CoverInput& in;
  signals::CoverPlan plan;
  std::vector<std::vector<uint32_t>> covers;
  std::map<std::string, uint32_t> held;      // process -> planned groups
  std::map<std::string, uint32_t> group_at;  // spans key -> index in plan.groups
  std::set<std::string> named;               // sets already in the plan (by members key)

  explicit Builder(const CoverInput& i) : in(i) {
    for (auto& [seat, n] : in.elsewhere) held["S" + seat.first + ":" + std::to_string(seat.second)] = n;
  }

  // A set's pipeline groups: per tensor column, the column's members in stage order.
  std::vector<std::vector<signals::SetMember>> groups_of(const std::vector<signals::SetMember>& members) const {
    std::vector<std::vector<signals::SetMember>> out;
    if (in.pp <= 1) return out;
    for (uint32_t col = 0; col < in.tp; col++) {
      std::vector<signals::SetMember> spans;
      for (const auto& m : members)
        if (position_of(m) % in.tp == col) spans.push_back(m);
      std::sort(spans.begin(), spans.end(),
                [&](const signals::SetMember& a, const signals::SetMember& b) { return position_of(a) < position_of(b); });
      if (spans.size() > 1) out.push_back(spans);
    }
    return out;
  }

  // Whether the set's new groups keep every process within the budget.
  bool fits(const std::vector<signals::SetMember>& members) const {
    if (in.max_groups_per_gpu == 0) return true;
    std::map<std::string, uint32_t> add;
    for (auto& g : groups_of(members))
      if (!group_at.count(spans_key(g)))
        for (auto& m : g) add[process_of(m)]++;
    for (auto& [p, n] : add) {
      auto it = held.find(p);
      if ((it == held.end() ? 0 : it->second) + n > in.max_groups_per_gpu) return false;
    }
    return true;
  }

  void admit(const std::vector<signals::SetMember>& members, const std::string& purpose,
             const std::vector<uint32_t>& lost) {
    signals::CoverSet set;
    set.members = members;
    set.purpose = purpose;
    for (auto& g : groups_of(members)) {
      const std::string k = spans_key(g);
      auto it = group_at.find(k);
      if (it == group_at.end()) {
        for (auto& m : g) held[process_of(m)]++;
        signals::CoverGroup cg;
        cg.scope = signals::Scope_SCOPE_FABRIC;
        cg.spans = g;
        cg.server = g.front();
        cg.has_server = true;
        it = group_at.emplace(k, (uint32_t)plan.groups.size()).first;
        plan.groups.push_back(cg);
      }
      set.groups.push_back(it->second);
    }
    named.insert(spans_key(members));
    plan.sets.push_back(set);
    covers.push_back(lost);
  }

  // Admit the set unless the plan holds it already; false when the budget refuses it.
  bool consider(const std::vector<signals::SetMember>& members, const std::string& purpose,
                const std::vector<uint32_t>& lost) {
    if (named.count(spans_key(members))) return true;
    if (!fits(members)) return false;
    admit(members, purpose, lost);
    return true;
  }

  uint32_t held_by(const SpareSeat& s) const {
    auto it = held.find("S" + s.node + ":" + std::to_string(s.device));
    return it == held.end() ? 0 : it->second;
  }

  // The REPLACE set for `lost`, or an empty vector when the spares cannot take every position.
  std::vector<signals::SetMember> replacement(const std::vector<uint32_t>& lost, const std::set<Seat>& exclude) const {
    const uint32_t world = in.tp * in.pp;
    // nodes the loss takes whole: a spare there dies with them
    std::set<std::string> gone;
    for (uint32_t r : lost) {
      auto h = in.holders.find(r);
      if (h == in.holders.end()) continue;
      bool whole = true;
      for (auto& [q, hq] : in.holders)
        if (hq.first == h->second.first && std::find(lost.begin(), lost.end(), q) == lost.end()) whole = false;
      if (whole) gone.insert(h->second.first);
    }
    std::set<Seat> taken;
    std::map<uint32_t, const SpareSeat*> by_rank;
    auto usable = [&](const SpareSeat& s) {
      const Seat seat{s.node, s.device};
      return !gone.count(s.node) && !exclude.count(seat) && !taken.count(seat);
    };
    for (uint32_t r : lost) {
      const SpareSeat* pick = nullptr;
      for (const auto& s : in.spares)
        if (s.for_rank == (int64_t)r && usable(s)) {
          pick = &s;
          break;
        }
      if (pick == nullptr) {
        for (const auto& s : in.spares)
          if (s.for_rank < 0 && usable(s) && (pick == nullptr || held_by(s) < held_by(*pick))) pick = &s;
      }
      if (pick == nullptr) return {};
      taken.insert({pick->node, pick->device});
      by_rank[r] = pick;
    }
    std::vector<signals::SetMember> members;
    for (uint32_t p = 0; p < world; p++) {
      auto it = by_rank.find(p);
      members.push_back(it == by_rank.end() ? rank_member(p) : spare_member(p, *it->second));
    }
    return members;
  }
};

std::string ranks_text(const std::vector<uint32_t>& lost) {
  std::string s = "[";
  for (size_t i = 0; i < lost.size(); i++) s += (i ? ", " : "") + std::to_string(lost[i]);
  return s + "]";
}

}  // namespace

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

std::vector<std::vector<uint32_t>> losses_of(const std::map<uint32_t, std::pair<std::string, uint32_t>>& holders) {
  std::map<std::string, std::vector<uint32_t>> by_node;
  for (auto& [r, h] : holders) by_node[h.first].push_back(r);
  std::vector<std::vector<uint32_t>> out;
  for (auto& [node, ranks] : by_node) out.push_back(ranks);
  for (auto& [node, ranks] : by_node)
    if (ranks.size() > 1)
      for (uint32_t r : ranks) out.push_back({r});
  return out;
}

bool answers(const std::vector<signals::SetMember>& members, const std::vector<uint32_t>& lost) {
  if (lost.empty()) return false;
  auto is_lost = [&](uint32_t p) { return std::find(lost.begin(), lost.end(), p) != lost.end(); };
  bool any_present = false, all_present = true;
  std::set<uint32_t> positions;
  for (const auto& m : members) {
    const uint32_t p = position_of(m);
    positions.insert(p);
    if (is_lost(p) && !m.has_spare) return false;  // a lost rank still serving
    if (!is_lost(p) && m.has_spare) return false;  // a survivor's position handed to a spare
  }
  for (uint32_t r : lost) {
    if (positions.count(r))
      any_present = true;
    else
      all_present = false;
  }
  return all_present || !any_present;  // every lost position replaced, or every one gone
}

signals::CoverPlan plan_cover(const CoverInput& in, std::vector<std::vector<uint32_t>>* covers,
                              std::vector<Uncovered>* uncovered) {
  Builder b(in);
  b.plan.engine = in.engine;
  b.plan.epoch = in.epoch;
  const uint32_t world = in.tp * in.pp;
  for (auto& [r, h] : in.holders) {
    signals::Holder ho;
    ho.node = h.first;
    ho.device = h.second;
    b.plan.placement[r] = ho;
  }
  {
    std::vector<signals::SetMember> current;
    for (uint32_t r = 0; r < world; r++) current.push_back(rank_member(r));
    b.admit(current, "current", {});
  }
  const auto losses = losses_of(in.holders);
  std::set<std::vector<uint32_t>> over_budget;
  for (const auto& lost : losses) {
    if (in.replace) {
      auto set = b.replacement(lost, {});
      if (!set.empty() && !b.consider(set, "REPLACE of ranks " + ranks_text(lost), lost)) over_budget.insert(lost);
    }
    if (in.shrink) {
      std::vector<signals::SetMember> survivors;
      for (uint32_t r = 0; r < world; r++)
        if (std::find(lost.begin(), lost.end(), r) == lost.end()) survivors.push_back(rank_member(r));
      if (!b.consider(survivors, "SHRINK of ranks " + ranks_text(lost), lost)) over_budget.insert(lost);
    }
  }
  if (in.replace) {
    for (const auto& lost : losses) {
      if (lost.size() != 1) continue;
      std::set<Seat> used;
      for (const auto& s : b.plan.sets)
        if (answers(s.members, lost))
          for (const auto& m : s.members)
            if (m.has_spare) used.insert({m.spare.node, m.spare.device});
      if (used.empty()) continue;
      auto set = b.replacement(lost, used);
      if (!set.empty() && !b.consider(set, "REPLACE of ranks " + ranks_text(lost) + " through a second spare", lost))
        over_budget.insert(lost);
    }
  }
  if (uncovered) {
    for (const auto& lost : losses) {
      bool covered = false;
      for (const auto& s : b.plan.sets) covered = covered || answers(s.members, lost);
      if (covered) continue;
      Uncovered u;
      u.lost = lost;
      if (over_budget.count(lost))
        u.why = "over the cover budget of " + std::to_string(in.max_groups_per_gpu) + " groups per GPU";
      else if (!in.replace && !in.shrink)
        u.why = "the policy allows neither REPLACE nor SHRINK";
      else
        u.why = "no spare can take it and SHRINK is not allowed";
      uncovered->push_back(u);
    }
  }
  if (covers) *covers = b.covers;
  return b.plan;
}

}  // namespace es
