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
  if (const Json* o = j.field("outcomesInOrder"))
    for (auto& v : o->arr) out.outcomes.push_back(outcome_of(v));
  if (out.outcomes.empty()) out.outcomes = {signals::Outcome_OUTCOME_REPLACE};
  out.max_concurrent_losses = u32(j.field("maxConcurrentLosses"), 0);
  out.notice_min_ms = u32(j.field("noticeMinMs"), 0);
  if (const Json* cv = j.field("cover")) {
    if (const Json* en = cv->field("enabled")) out.cover_enabled = en->b;
    out.cover_max_groups_per_gpu = u32(cv->field("maxGroupsPerGpu"), 0);
  }
  if (const Json* sp = j.field("spares")) {
    out.spares.per_engine = u32(sp->field("perEngine"), 0);
    if (const Json* l = sp->field("loading"))
      out.spares.loading = l->kind == Json::Number ? (int32_t)l->num
                           : l->str == "LOADING_PRELOADED" ? 1 : l->str == "LOADING_ON_NOTICE" ? 2 : 0;
    if (const Json* am = sp->field("allowMismatched")) out.spares.allow_mismatched = am->b;
    out.spares.max_degrade_percent = u32(sp->field("maxDegradePercent"), 0);
  }
  if (const Json* es = j.field("engines")) {
    for (auto& e : es->arr) {
      EnginePolicy ep;
      if (const Json* n = e.field("name")) ep.name = n->str;
      if (ep.name.empty()) {
        err = "an engine without a name";
        return false;
      }
      ep.tensor = std::max<uint32_t>(1, u32(e.field("tensorParallel"), 1));
      ep.pipeline = std::max<uint32_t>(1, u32(e.field("pipelineParallel"), 1));
      ep.data = std::max<uint32_t>(1, u32(e.field("dataParallel"), 1));
      ep.expert = std::max<uint32_t>(1, u32(e.field("expertParallel"), 1));
      if (const Json* pi = e.field("placementIndependentModel")) ep.placement_independent = pi->b;
      if (const Json* sn = e.field("spareNodes"))
        for (auto& s : sn->arr) ep.spare_nodes.push_back(s.str);
      if (const Json* rb = e.field("releaseBoundMs")) ep.release_bound_ms = (int64_t)u32(rb, 0);
      if (const Json* rn = e.field("replicaNodes"))
        for (auto& n : rn->arr) ep.replica_nodes.push_back(n.str);
      if (const Json* sl = e.field("spares"))
        for (auto& x : sl->arr) {
          SpareSlotPolicy slot;
          if (const Json* n = x.field("node")) slot.node = n->str;
          slot.device = u32(x.field("device"), 0);
          if (const Json* r = x.field("rank")) slot.rank = (int64_t)u32(r, 0);
          ep.spare_slots.push_back(slot);
        }
      if (const Json* sl = e.field("spareLaunch")) {
        if (const Json* c = sl->field("command"))
          for (auto& a : c->arr) ep.launch_command.push_back(a.str);
        if (const Json* env = sl->field("env"))
          for (auto& [k, v] : env->obj) ep.launch_env[k] = v.str;
      }
      out.engines[ep.name] = ep;
    }
  }
  return true;
}

bool parse_pool(const std::string& json, PoolSpec& out, std::string& err) {
  Json j;
  if (!Json::parse(json, j, &err)) return false;
  if (j.kind != Json::Object) {
    err = "a pool spec is a JSON object";
    return false;
  }
  out = PoolSpec{};
  if (const Json* n = j.get("name")) out.name = n->str;
  if (const Json* es = j.get("engines"))
    for (auto& e : es->arr) out.engines.push_back(e.str);
  out.wants = u32(j.get("wants"), 0);
  if (const Json* c = j.get("deviceClass")) out.device_class = c->str;
  if (const Json* d = j.get("domain")) out.domain = d->str;
  if (const Json* r = j.get("reason")) out.reason = r->str;
  if (const Json* c = j.get("command"))
    for (auto& a : c->arr) out.command.push_back(a.str);
  if (const Json* env = j.get("env"))
    for (auto& [k, v] : env->obj) out.env[k] = v.str;
  if (const Json* g = j.get("generation")) out.generation = g->kind == Json::Number ? (uint64_t)g->num : std::stoull(g->str);
  return true;
}

std::string pool_json(const PoolSpec& p) {
  auto list = [](const std::vector<std::string>& v) {
    std::string o = "[";
    for (size_t i = 0; i < v.size(); i++) o += (i ? ",\"" : "\"") + json_escape(v[i]) + "\"";
    return o + "]";
  };
  std::string env = "{";
  bool first = true;
  for (auto& [k, v] : p.env) {
    env += std::string(first ? "" : ",") + "\"" + json_escape(k) + "\":\"" + json_escape(v) + "\"";
    first = false;
  }
  env += "}";
  return "{\"name\":\"" + json_escape(p.name) + "\",\"engines\":" + list(p.engines) + ",\"wants\":" +
         std::to_string(p.wants) + ",\"deviceClass\":\"" + json_escape(p.device_class) + "\",\"domain\":\"" +
         json_escape(p.domain) + "\",\"reason\":\"" + json_escape(p.reason) + "\",\"command\":" + list(p.command) +
         ",\"env\":" + env + ",\"generation\":" + std::to_string(p.generation) + "}";
}

std::vector<std::pair<std::string, uint32_t>> place_pool_spares(const PoolSpec& pool,
                                                                 const std::vector<FreeDevice>& free, uint32_t count) {
  std::map<std::string, std::vector<uint32_t>> by_node;
  for (auto& d : free) {
    if (!pool.device_class.empty() && d.cls.find(pool.device_class) == std::string::npos) continue;
    if (!pool.domain.empty() && d.domain != pool.domain) continue;
    by_node[d.node].push_back(d.device);
  }
  for (auto& [n, devs] : by_node) std::sort(devs.begin(), devs.end());
  std::vector<std::pair<std::string, uint32_t>> out;
  for (size_t round = 0; out.size() < count; round++) {
    bool any = false;
    for (auto& [n, devs] : by_node) {
      if (round >= devs.size() || out.size() >= count) continue;
      out.emplace_back(n, devs[round]);
      any = true;
    }
    if (!any) break;
  }
  return out;
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
