#include "state.h"

#include <algorithm>

#include "everserve_pb.h"

namespace es {

uint32_t Policy::world_size(const std::string& engine) const {
  auto it = engines.find(engine);
  if (it == engines.end()) return 0;
  return it->second.tensor * it->second.pipeline * it->second.data;
}

static int32_t outcome_of(const Json& v) {
  if (v.kind == Json::Number) return (int32_t)v.num;
  if (v.str == "OUTCOME_REPLACE") return signals::Outcome_OUTCOME_REPLACE;
  if (v.str == "OUTCOME_SHRINK") return signals::Outcome_OUTCOME_SHRINK;
  if (v.str == "OUTCOME_REBUILD") return signals::Outcome_OUTCOME_REBUILD;
  return 0;
}

static uint32_t u32(const Json* v, uint32_t dflt) {
  if (v == nullptr) return dflt;
  if (v->kind == Json::Number) return (uint32_t)v->num;
  if (v->kind == Json::String) return (uint32_t)std::stoul(v->str);
  return dflt;
}

bool parse_policy(const std::string& json, Policy& out, std::string& err) {
  Json j;
  if (!Json::parse(json, j, &err)) return false;
  if (j.kind != Json::Object) {
    err = "the policy is not a JSON object";
    return false;
  }
  out = Policy{};
  if (const Json* o = j.get("outcomesInOrder"))
    for (auto& v : o->arr) out.outcomes.push_back(outcome_of(v));
  if (out.outcomes.empty()) out.outcomes = {signals::Outcome_OUTCOME_REPLACE};
  out.max_concurrent_losses = u32(j.get("maxConcurrentLosses"), 0);
  out.notice_min_ms = u32(j.get("noticeMinMs"), 0);
  if (const Json* cv = j.get("cover")) {
    if (const Json* en = cv->get("enabled")) out.cover_enabled = en->b;
    out.cover_max_groups_per_gpu = u32(cv->get("maxGroupsPerGpu"), 0);
  }
  if (const Json* es = j.get("engines")) {
    for (auto& e : es->arr) {
      EnginePolicy ep;
      if (const Json* n = e.get("name")) ep.name = n->str;
      if (ep.name.empty()) {
        err = "an engine without a name";
        return false;
      }
      ep.tensor = std::max<uint32_t>(1, u32(e.get("tensorParallel"), 1));
      ep.pipeline = std::max<uint32_t>(1, u32(e.get("pipelineParallel"), 1));
      ep.data = std::max<uint32_t>(1, u32(e.get("dataParallel"), 1));
      ep.expert = std::max<uint32_t>(1, u32(e.get("expertParallel"), 1));
      if (const Json* pi = e.get("placementIndependentModel")) ep.placement_independent = pi->b;
      if (const Json* sn = e.get("spareNodes"))
        for (auto& s : sn->arr) ep.spare_nodes.push_back(s.str);
      if (const Json* rb = e.get("releaseBoundMs")) ep.release_bound_ms = (int64_t)u32(rb, 0);
      if (const Json* rn = e.get("replicaNodes"))
        for (auto& n : rn->arr) ep.replica_nodes.push_back(n.str);
      if (const Json* sl = e.get("spares"))
        for (auto& x : sl->arr) {
          SpareSlotPolicy slot;
          if (const Json* n = x.get("node")) slot.node = n->str;
          slot.device = u32(x.get("device"), 0);
          if (const Json* r = x.get("rank")) slot.rank = (int64_t)u32(r, 0);
          ep.spare_slots.push_back(slot);
        }
      if (const Json* sl = e.get("spareLaunch")) {
        if (const Json* c = sl->get("command"))
          for (auto& a : c->arr) ep.launch_command.push_back(a.str);
        if (const Json* env = sl->get("env"))
          for (auto& [k, v] : env->obj) ep.launch_env[k] = v.str;
      }
      out.engines[ep.name] = ep;
    }
  }
  return true;
}

Choice choose_outcome(const Policy& p, const std::string& engine, const std::set<uint32_t>& lost,
                      const std::vector<SpareSeat>& spares, const std::string& fingerprint) {
  Choice c;
  if (p.max_concurrent_losses && lost.size() > p.max_concurrent_losses) {
    c.why = "more concurrent losses than the policy allows";
    return c;
  }
  auto ep = p.engines.find(engine);
  for (int32_t want : p.outcomes) {
    if (want == signals::Outcome_OUTCOME_REPLACE) {
      std::vector<bool> used(spares.size(), false);
      for (size_t i = 0; i < spares.size(); i++)  // another build cannot take a rank exactly
        if (!fingerprint.empty() && !spares[i].fingerprint.empty() && spares[i].fingerprint != fingerprint)
          used[i] = true;
      std::vector<std::pair<uint32_t, SpareSeat>> take;
      bool all = true;
      for (uint32_t r : lost) {
        int pick = -1;
        for (size_t i = 0; i < spares.size() && pick < 0; i++)
          if (!used[i] && spares[i].for_rank == (int64_t)r) pick = (int)i;
        for (size_t i = 0; i < spares.size() && pick < 0; i++)
          if (!used[i] && spares[i].for_rank < 0) pick = (int)i;
        if (pick < 0) {
          all = false;
          break;
        }
        used[(size_t)pick] = true;
        take.emplace_back(r, spares[(size_t)pick]);
      }
      if (all) {
        c.outcome = want;
        c.take = std::move(take);
        return c;
      }
      c.why = "no spare for every lost rank";
    } else if (want == signals::Outcome_OUTCOME_SHRINK) {
      if (ep != p.engines.end() && ep->second.placement_independent) {
        c.outcome = want;
        return c;
      }
      c.why += (c.why.empty() ? "" : "; ") + std::string("shrink needs a placement-independent model");
    } else if (want == signals::Outcome_OUTCOME_REBUILD) {
      c.why += (c.why.empty() ? "" : "; ") + std::string("rebuild restarts the engine");
    }
  }
  return c;
}

}  // namespace es
