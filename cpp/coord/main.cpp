// everserve-coord: the coordinator, the single writer of membership epochs (one per cluster).
//
//   everserve-coord --listen unix:/run/everserve/coord.sock --policy policy.json --spec-store DIR
//                   [--lease FILE] [--api-addr host:port] [--metrics-addr host:port]
//                   [--node-loss-misses 3] [--delivery-timeout-ms 130000] [--fold-ms 3]
//                   [--lease-holder NAME] [--lease-duration-s 15]   (--lease k8s:NS/NAME: a Kubernetes Lease)
//                   [--enroll-addr host:port] [--enroll-ca-dir DIR] [--enroll-hours 12]   (node enrollment, issuer.h)
//                   [--api-auth cert|kube] [--api-namespace NS]   (operator API: client certificates, or api_auth.h)
// Flags also read EVERSERVE_LISTEN, EVERSERVE_POLICY, EVERSERVE_SPEC_STORE, EVERSERVE_LEASE,
// EVERSERVE_API_ADDR, EVERSERVE_METRICS_ADDR, EVERSERVE_NODE_LOSS_MISSES.
//
// Node daemons link to it (coord.proto). From their hellos and worker events it keeps a view of
// every engine: its epoch, which node holds each rank, and the spares. A loss (a rank reported
// lost, a worker connection that ended, a node whose heartbeats stopped) folds into the engine's
// pending losses; the transition machine then
//   claim    -> chooses the outcome by policy (REPLACE with a spare per lost rank, ...), epoch + 1,
//   log      -> writes the change to the spec store BEFORE any node hears of it,
//   deliver  -> one Deliver per node (its surviving ranks, its spares that take ranks),
//   acks     -> every node answers Delivered with its processes' acks (bounded),
//   commit   -> MembershipCommitted to every node of the engine, and the spec store is updated;
// any failure on the way abandons the change (the engine is down; its processes are told).
// A lease (a locked file holding the term) makes this process the writer; every message to a
// daemon carries the term, and daemons ignore older terms. On start, a change logged but not
// committed by an earlier holder is delivered again once the daemons have linked.
#include <fcntl.h>
#include <signal.h>
#include <sys/file.h>
#include <unistd.h>

#include <algorithm>
#include <deque>
#include <map>
#include <set>
#include <thread>

#include "cover.h"
#include "everserve_pb.h"
#include "api_auth.h"
#include "issuer.h"
#include "lease.h"
#include "spec_store.h"
#include "topology.h"
#include "net.h"
#include "state.h"
#include "telemetry.h"
#include "tls.h"
#include "util.h"

using namespace es;

namespace {

struct Holder {
  std::string node;
  uint32_t device = 0;
  uint32_t pid = 0;
  std::string host;
  signals::CompileCache cache;  // the compile-cache pair its worker registered
};

struct InFlight {
  signals::Change change;
  std::string cause;
  std::map<std::string, coord::Deliver> deliveries;  // node -> what it was sent
  std::set<std::string> waiting;                      // nodes that owe Delivered
  std::vector<signals::Ack> acks;
  uint64_t reported_us = 0, delivered_us = 0, started_ms = 0;
  std::vector<std::pair<uint32_t, SpareSeat>> take;
};

struct Engine {
  std::string name;
  std::string fingerprint;  // the first worker's identity fingerprint
  uint64_t epoch = 0;
  uint32_t world = 0;
  std::map<uint32_t, Holder> workers;
  std::vector<SpareSeat> spares;  // the admitted spares, in node and device order
  // every spare that registered, by (node, device), and why those not admitted are refused
  std::map<std::pair<std::string, uint32_t>, SpareSeat> standing;
  std::map<std::pair<std::string, uint32_t>, std::string> refused;
  std::set<std::string> head_nodes;
  std::set<std::string> listeners;  // nodes where a process asked for the engine's start-up record
  std::deque<double> pauses_ms;     // the last changes' pauses (report to commit), newest last
  bool drive_posted = false;        // a drive is queued behind the reports now being read
  std::set<uint32_t> pending;
  std::set<uint32_t> departing;  // planned departures among pending
  uint64_t first_report_us = 0;
  std::string cause;
  bool down = false;
  std::unique_ptr<InFlight> in_flight;
  // the cover plan last sent, and which members reported each planned group formed
  uint64_t cover_gen = 0;
  std::string cover_sig;
  signals::CoverPlan cover;
  std::vector<std::vector<uint32_t>> cover_covers;
  std::vector<Uncovered> cover_uncovered;  // losses the plan leaves unanswered, with the reason
  std::map<std::string, std::set<std::string>> cover_formed;
  std::map<std::string, std::string> cover_failed;
  // a change an earlier lease holder logged but did not commit: finished once its nodes link
  bool has_resume = false;
  spec::ChangeLog resume;
  std::map<uint32_t, std::vector<std::string>> replicas;  // rank -> replica stores last asked for
};

struct Node {
  std::string name;
  std::string replica_address;  // the node's store, for rows replicated to it
  uint64_t conn = 0;
  uint64_t last_seen_ms = 0;
  uint32_t heartbeat_ms = 500;
  bool linked = false;
  bool cordoned = false;
  int64_t drain_by_ms = 0;
};

struct Event {
  uint64_t seq;
  uint64_t at_ms;
  std::string text;
  std::string engine;  // the engine it concerns ("" for node events)
};

struct Coordinator {
  Loop loop;
  Policy policy;
  std::string spec_dir;               // the --spec-store flag
  std::unique_ptr<SpecStore> spec;    // nullptr: nothing outlives this process
  uint64_t term = 1;
  uint32_t loss_misses = 3;
  uint64_t delivery_timeout_ms = 130000;
  uint64_t fold_ms = 3;  // how long a first loss report waits for others to fold into its change
  bool exit_after_log = false;  // host-side fault injection for tests: the coordinator dies mid-change
  std::map<std::string, Engine> engines;
  std::map<std::string, Node> nodes;
  std::map<uint64_t, std::string> conn_node;
  uint64_t next_request = 1;
  std::deque<Event> events;
  uint64_t event_seq = 0;
  // stack dumps by request: (node, pid) -> text, kept for the last 64 requests
  std::map<uint64_t, std::vector<std::pair<std::string, std::string>>> stacks;
  Topology topo;  // every node's devices, from the daemons' hellos
  std::map<std::string, PoolSpec> pools;
  // pool spares launched and not yet registered: (node, device) -> (pool, launched at ms)
  std::map<std::pair<std::string, uint32_t>, std::pair<std::string, uint64_t>> pool_launches;
  uint64_t pool_warm_ms = 600000;  // a launch not registered within this is tried elsewhere

  void event(const std::string& text) {
    std::string eng;
    if (text.rfind("engine ", 0) == 0) eng = text.substr(7, text.find(':') == std::string::npos ? 0 : text.find(':') - 7);
    events.push_back({++event_seq, now_ms(), text, eng});
    if (events.size() > 4096) events.pop_front();
    ES_INFO("%s", text.c_str());
  }

  Engine& engine(const std::string& name) {
    Engine& e = engines[name];
    if (e.name.empty()) {
      e.name = name;
      e.world = policy.world_size(name);
    }
    return e;
  }

  void to_node(const std::string& node, coord::CoordToDaemon& m) {
    auto it = nodes.find(node);
    if (it == nodes.end() || !it->second.linked) return;
    m.term = term;
    loop.send(it->second.conn, m.serialize());
  }

  std::set<std::string> engine_nodes(const Engine& e) {
    std::set<std::string> out = e.head_nodes;
    for (auto& [r, h] : e.workers) out.insert(h.node);
    for (auto& s : e.spares) out.insert(s.node);
    return out;
  }

  // ---- spec store ------------------------------------------------------------------------------
  void write_status(const Engine& e, const InFlight* f, const coord::Committed* committed) {
    if (!spec) return;
    spec::EngineStatus st;
    st.engine = e.name;
    for (auto& [r, h] : e.workers) {
      spec::Assignment a;
      a.rank = r;
      a.epoch = e.epoch;
      a.node = h.node;
      a.host = h.host;
      st.assignments.push_back(a);
    }
    if (f != nullptr) {
      st.has_change = true;
      st.change.change = f->change;
      st.change.has_change = true;
      st.change.world_size = e.world;
      st.change.taking = f->change.take;
      for (auto& [node, d] : f->deliveries) {
        spec::NodeDelivery nd;
        nd.node = node;
        nd.to_ranks = d.to_ranks;
        nd.to_spares = d.to_spares;
        nd.take = d.take;
        st.change.deliveries.push_back(nd);
      }
      if (committed != nullptr) {
        st.change.committed = *committed;
        st.change.has_committed = true;
      }
    }
    if (!spec->put(e.name + ".status", st.serialize()))
      ES_ERROR("cannot write the spec store at %s", spec->where().c_str());
    metrics().inc("everserve_spec_writes_total");
  }

  void write_node(const Node& n) {
    if (!spec) return;
    const std::string j = "{\"node\":\"" + json_escape(n.name) + "\",\"unschedulable\":" +
                          (n.cordoned ? "true" : "false") + ",\"drainByMs\":" + std::to_string(n.drain_by_ms) + "}";
    if (!spec->put("nodes/" + n.name + ".json", j)) ES_ERROR("cannot write node %s's spec", n.name.c_str());
    metrics().inc("everserve_spec_writes_total", {{"kind", "node"}, {"verdict", "written"}});
  }

  void load_nodes() {
    std::map<std::string, std::string> all;
    if (!spec || !spec->list("nodes/", all)) return;
    for (auto& [key, text] : all) {
      Json j;
      std::string err;
      if (!Json::parse(text, j, &err)) continue;
      const Json* name = j.get("node");
      if (!name || name->str.empty()) continue;
      Node& n = nodes[name->str];
      n.name = name->str;
      if (const Json* u = j.get("unschedulable")) n.cordoned = u->b;
      if (const Json* d = j.get("drainByMs")) n.drain_by_ms = (int64_t)d->num;
    }
  }

  // ---- the transition machine ------------------------------------------------------------------
  void report_loss(const std::string& name, const std::vector<uint32_t>& ranks, uint64_t epoch, const std::string& cause,
                   bool planned = false) {
    Engine& e = engine(name);
    if (epoch != 0 && epoch < e.epoch) {
      metrics().inc("everserve_fenced_total");
      return;  // a report from before the last change: stale
    }
    bool any = false;
    for (uint32_t r : ranks) {
      if (!e.workers.count(r)) {
        metrics().inc("everserve_unheard_ranks_lost_total");
        continue;
      }
      if (e.pending.insert(r).second) any = true;
      if (planned) e.departing.insert(r);
    }
    if (!any) return;
    if (e.first_report_us == 0) e.first_report_us = now_us();
    e.cause = cause;
    event("engine " + name + ": lost ranks reported (" + cause + ")");
    // the change starts `fold_ms` after the first report: losses that arrive together (processes
    // of one node dying within a scan or two of its daemon's watcher) fold into one change rather
    // than one change meeting the next loss in flight
    if (!e.drive_posted) {
      e.drive_posted = true;
      auto go = [this, name] {
        Engine& en = engine(name);
        en.drive_posted = false;
        drive(en);
      };
      if (fold_ms == 0) loop.post(go);
      else loop.every(fold_ms, go, false);
    }
  }

  void drive(Engine& e) {
    if (e.in_flight || e.pending.empty() || e.down) return;
    const uint64_t t0 = now_us();
    Choice c = choose_outcome(policy, e.name, e.pending, e.spares, e.fingerprint);
    metrics().observe("everserve_change_decision_seconds", {{"engine", e.name}}, (now_us() - t0) * 1e-6);
    if (c.outcome == 0) {
      abandon(e, "no outcome: " + c.why);
      return;
    }
    auto f = std::make_unique<InFlight>();
    f->change.epoch = e.epoch + 1;
    f->change.outcome = c.outcome;
    f->change.lost.assign(e.pending.begin(), e.pending.end());
    f->change.departing.assign(e.departing.begin(), e.departing.end());
    f->cause = e.cause;
    f->take = c.take;
    for (auto& [rank, seat] : c.take) {
      signals::Take t;
      t.rank = rank;
      t.node = seat.node;
      t.device = seat.device;
      f->change.take.push_back(t);
    }
    f->reported_us = e.first_report_us;
    f->started_ms = now_ms();
    // one delivery per node: its surviving (or departing) ranks and its taking spares
    for (auto& [r, h] : e.workers) {
      const bool lost_now = e.pending.count(r) && !e.departing.count(r);
      if (lost_now) continue;
      auto& d = f->deliveries[h.node];
      d.to_ranks.push_back(r);
    }
    for (auto& [rank, seat] : c.take) {
      auto& d = f->deliveries[seat.node];
      d.to_spares.push_back(rank);
      signals::Take t;
      t.rank = rank;
      t.node = seat.node;
      t.device = seat.device;
      d.take.push_back(t);
    }
    for (auto& hn : e.head_nodes) f->deliveries[hn];  // the head hears the change on its node
    for (auto& [node, d] : f->deliveries) {
      d.request_id = next_request++;
      d.engine = e.name;
      d.change = f->change;
      d.has_change = true;
    }
    // logged before any node hears of it
    write_status(e, f.get(), nullptr);
    if (exit_after_log) {
      ES_WARN("exiting after logging the change (EVERSERVE_COORD_EXIT_AFTER_LOG)");
      _exit(17);
    }
    e.pending.clear();
    e.departing.clear();
    e.first_report_us = 0;
    start_delivery(e, std::move(f));
  }

  // Deliver a logged change to every node it names and wait for their acks (bounded).
  void start_delivery(Engine& e, std::unique_ptr<InFlight> f) {
    f->delivered_us = now_us();
    for (auto& [node, d] : f->deliveries) {
      auto nit = nodes.find(node);
      if (nit == nodes.end() || !nit->second.linked) {
        e.in_flight = std::move(f);
        abandon(e, "node " + node + " is not linked");
        return;
      }
      f->waiting.insert(node);
      coord::CoordToDaemon m;
      m.has_deliver = true;
      m.deliver = d;
      to_node(node, m);
    }
    metrics().set("everserve_changes_in_flight", {{"engine", e.name}}, 1);
    event("engine " + e.name + ": change to epoch " + std::to_string(f->change.epoch) + " delivered to " +
          std::to_string(f->deliveries.size()) + " node(s)");
    e.in_flight = std::move(f);
    const std::string name = e.name;
    const uint64_t epoch = e.in_flight->change.epoch;
    loop.every(delivery_timeout_ms, [this, name, epoch] {
      Engine& en = engines[name];
      if (en.in_flight && en.in_flight->change.epoch == epoch) abandon(en, "acks timed out");
    }, false);
    if (e.in_flight->waiting.empty()) commit(e);
  }

  void delivered(const std::string& node, const coord::Delivered& d) {
    auto it = engines.find(d.engine);
    if (it == engines.end() || !it->second.in_flight) return;
    Engine& e = it->second;
    InFlight& f = *e.in_flight;
    if (d.epoch != f.change.epoch || !f.waiting.count(node)) return;
    for (auto& a : d.acks) f.acks.push_back(a);
    if (!d.error.empty()) {
      abandon(e, "node " + node + ": " + d.error);
      return;
    }
    f.waiting.erase(node);
    if (f.waiting.empty()) commit(e);
  }

  void commit(Engine& e) {
    InFlight& f = *e.in_flight;
    const uint64_t acked_us = now_us();
    // the new membership: lost ranks leave, the spares that took them hold them
    for (uint32_t r : f.change.lost) e.workers.erase(r);
    for (auto& [rank, seat] : f.take) {
      Holder h;
      h.node = seat.node;
      h.device = seat.device;
      h.pid = seat.pid;
      e.workers[rank] = h;
      e.spares.erase(std::remove_if(e.spares.begin(), e.spares.end(),
                                    [&](const SpareSeat& s) { return s.node == seat.node && s.device == seat.device; }),
                     e.spares.end());
      e.standing.erase({seat.node, seat.device});
      e.refused.erase({seat.node, seat.device});
      // a pool spare stands for every engine of its pool: once one takes it, the others lose it
      for (auto& [oname, other] : engines)
        if (&other != &e && other.standing.erase({seat.node, seat.device})) admit(other);
    }
    e.epoch = f.change.epoch;
    coord::Committed c;
    c.engine = e.name;
    c.outcome = f.change.outcome;
    c.lost = f.change.lost;
    c.take = f.change.take;
    c.has_membership = true;
    auto& mc = c.membership;
    mc.epoch = e.epoch;
    for (auto& [r, h] : e.workers) {
      mc.active_ranks.push_back(r);
      signals::RankPlacement p;
      p.rank = r;
      p.node = h.node;
      p.device = h.device;
      p.has_device = true;
      p.host = h.host;
      mc.members.push_back(p);
    }
    mc.world_size = e.world ? e.world : (uint32_t)e.workers.size();
    mc.lost = f.change.lost;
    mc.reported_at_us = f.reported_us;
    mc.delivered_at_us = f.delivered_us;
    mc.acknowledged_at_us = acked_us;
    mc.committed_at_us = now_us();
    mc.acks = f.acks;
    mc.pause_ms = (uint32_t)((mc.committed_at_us - (f.reported_us ? f.reported_us : f.delivered_us)) / 1000);
    e.pauses_ms.push_back((mc.committed_at_us - (f.reported_us ? f.reported_us : f.delivered_us)) / 1e3);
    if (e.pauses_ms.size() > 16) e.pauses_ms.pop_front();
    write_status(e, &f, &c);
    coord::CoordToDaemon m;
    m.has_committed = true;
    m.committed = c;
    for (auto& node : engine_nodes(e)) to_node(node, m);
    for (auto& [node, d] : f.deliveries)
      if (!engine_nodes(e).count(node)) to_node(node, m);
    const double secs = (mc.committed_at_us - (f.reported_us ? f.reported_us : f.delivered_us)) * 1e-6;
    metrics().inc("everserve_changes_total",
                  {{"engine", e.name}, {"cause", f.cause}, {"outcome", std::to_string(f.change.outcome)}, {"verdict", "committed"}});
    metrics().observe("everserve_change_seconds", {{"engine", e.name}}, secs);
    metrics().set("everserve_changes_in_flight", {{"engine", e.name}}, 0);
    event("engine " + e.name + ": epoch " + std::to_string(e.epoch) + " committed in " + std::to_string(secs * 1e3) +
          " ms");
    e.in_flight.reset();
    admit(e);
    update_gauges(&e);
    replan(e);
    replicate(e);
    reconcile_pools();
    send_placement(e);
    drive(e);  // losses that arrived during the change
  }

  void abandon(Engine& e, const std::string& why) {
    const uint64_t epoch = e.in_flight ? e.in_flight->change.epoch : e.epoch + 1;
    coord::CoordToDaemon m;
    m.has_abandon = true;
    m.abandon.engine = e.name;
    m.abandon.epoch = epoch;
    m.abandon.detail = why;
    std::set<std::string> targets = engine_nodes(e);
    if (e.in_flight)
      for (auto& [node, d] : e.in_flight->deliveries) targets.insert(node);
    for (auto& node : targets) to_node(node, m);
    metrics().inc("everserve_changes_total",
                  {{"engine", e.name}, {"cause", e.cause}, {"outcome", "0"}, {"verdict", "abandoned"}});
    metrics().set("everserve_changes_in_flight", {{"engine", e.name}}, 0);
    metrics().set("everserve_engine_down", {{"engine", e.name}}, 1);
    e.down = true;
    e.in_flight.reset();
    e.pending.clear();
    event("engine " + e.name + ": change abandoned, engine down: " + why);
    admit(e);
  }

  // The spare gauge of `only` (of every engine when `all`): per-engine gauges are set where that
  // engine changed, so an event costs O(1) metric writes whatever the fleet's size; the
  // fleet-wide gauges are refreshed on a timer (fleet_gauges).
  void update_gauges(const Engine* only = nullptr, bool all = false) {
    if (all)
      for (auto& [name, e] : engines)
        metrics().set("everserve_spares", {{"engine", name}, {"state", "standing"}}, (double)e.spares.size());
    else if (only != nullptr)
      metrics().set("everserve_spares", {{"engine", only->name}, {"state", "standing"}}, (double)only->spares.size());
  }

  void fleet_gauges() {
    uint64_t linked = 0, workers = 0;
    for (auto& [n, node] : nodes) linked += node.linked;
    for (auto& [name, e] : engines) workers += e.workers.size();
    metrics().set("everserve_daemons_connected", {}, (double)linked);
    metrics().set("everserve_workers_registered", {}, (double)workers);
  }

  // Whether `node` needs `e`'s placement (placement_nodes, by lookups rather than a full walk).
  bool needs_placement(const Engine& e, const std::string& node) const {
    if (e.head_nodes.count(node) || e.listeners.count(node)) return true;
    for (auto& [r, h] : e.workers)
      if (h.node == node) return true;
    auto st = e.standing.lower_bound({node, 0});
    if (st != e.standing.end() && st->first.first == node) return true;
    auto ep = policy.engines.find(e.name);
    if (ep != policy.engines.end())
      for (auto& slot : ep->second.spare_slots)
        if (slot.node == node) return true;
    return false;
  }

  // ---- takeover: views from the spec store and the daemons' announcements ----------------------
  void load_spec() {
    std::map<std::string, std::string> all;
    if (!spec || !spec->list("", all)) return;
    for (auto& [f, data] : all) {
      if (f.find('/') != std::string::npos || f.size() < 8 || f.compare(f.size() - 7, 7, ".status") != 0) continue;
      spec::EngineStatus st;
      if (!st.parse(data) || st.engine.empty()) continue;
      Engine& e = engine(st.engine);
      for (auto& a : st.assignments) e.epoch = std::max(e.epoch, a.epoch);
      if (st.has_change && st.change.has_change) {
        if (st.change.has_committed) {
          e.epoch = std::max(e.epoch, st.change.change.epoch);
        } else {
          e.has_resume = true;
          e.resume = st.change;
          e.epoch = std::max(e.epoch, st.change.change.epoch - 1);
          event("engine " + e.name + ": change to epoch " + std::to_string(st.change.change.epoch) +
                " was logged by the previous lease holder and is not committed; finishing it");
        }
      }
    }
  }

  void try_resume(Engine& e) {
    if (!e.has_resume || e.in_flight) return;
    for (auto& nd : e.resume.deliveries) {
      auto it = nodes.find(nd.node);
      if (it == nodes.end() || !it->second.linked) return;  // wait for every node it names
    }
    auto f = std::make_unique<InFlight>();
    f->change = e.resume.change;
    f->cause = "resumed";
    f->started_ms = now_ms();
    for (auto& t : e.resume.change.take) {
      SpareSeat seat;
      seat.node = t.node;
      seat.device = t.device;
      for (auto& sp : e.spares)
        if (sp.node == t.node && sp.device == t.device) seat = sp;
      f->take.emplace_back(t.rank, seat);
    }
    for (auto& nd : e.resume.deliveries) {
      coord::Deliver d;
      d.request_id = next_request++;
      d.engine = e.name;
      d.change = f->change;
      d.has_change = true;
      d.to_ranks = nd.to_ranks;
      d.to_spares = nd.to_spares;
      d.take = nd.take;
      f->deliveries[nd.node] = d;
    }
    e.has_resume = false;
    e.down = false;
    start_delivery(e, std::move(f));
  }

  // ---- replication: each rank's rows also go to the stores of the nodes that may restore it ---
  void replicate(Engine& e) {
    auto ep = policy.engines.find(e.name);
    for (auto& [r, h] : e.workers) {
      std::set<std::string> target_nodes;
      if (ep != policy.engines.end() && !ep->second.replica_nodes.empty()) {
        for (auto& n : ep->second.replica_nodes) target_nodes.insert(n);
      } else {
        for (auto& sp : e.spares)  // the nodes whose spares may take this rank
          if (sp.for_rank < 0 || sp.for_rank == (int64_t)r) target_nodes.insert(sp.node);
      }
      target_nodes.erase(h.node);
      std::vector<std::string> targets;
      for (auto& n : target_nodes) {
        auto it = nodes.find(n);
        if (it != nodes.end() && !it->second.replica_address.empty()) targets.push_back(it->second.replica_address);
      }
      if (e.replicas[r] == targets) continue;
      e.replicas[r] = targets;
      coord::CoordToDaemon m;
      m.has_replicate_targets = true;
      m.replicate_targets.engine = e.name;
      m.replicate_targets.rank = r;
      m.replicate_targets.targets = targets;
      to_node(h.node, m);
    }
  }

  // ---- placement: where each rank runs, its compile-cache pair and the stores that hold it -----
  // The nodes that need an engine's placement: its ranks', heads' and spares' nodes, and the
  // nodes where spares for it are launched (they fetch the engine's compile cache from it).
  std::set<std::string> placement_nodes(const Engine& e) {
    std::set<std::string> to = engine_nodes(e);
    for (auto& [key, seat] : e.standing) to.insert(key.first);
    to.insert(e.listeners.begin(), e.listeners.end());
    auto ep = policy.engines.find(e.name);
    if (ep != policy.engines.end())
      for (auto& slot : ep->second.spare_slots) to.insert(slot.node);
    for (auto& [key, launch] : pool_launches) {
      auto pit = pools.find(launch.first);
      if (pit != pools.end() &&
          std::find(pit->second.engines.begin(), pit->second.engines.end(), e.name) != pit->second.engines.end())
        to.insert(key.first);
    }
    return to;
  }

  void send_placement(const Engine& e, const std::string& only_node = "") {
    coord::CoordToDaemon m;
    m.has_engine_placement = true;
    auto& pl = m.engine_placement;
    pl.engine = e.name;
    pl.epoch = e.epoch;
    for (auto& [r, h] : e.workers) {
      signals::RankPlacement p;
      p.rank = r;
      p.node = h.node;
      p.device = h.device;
      p.has_device = true;
      p.host = h.host;
      if (!h.cache.key.empty()) {
        p.compile_cache = h.cache;
        p.has_compile_cache = true;
        std::set<std::string> holders;  // every node whose worker registered the same pair
        for (auto& [r2, h2] : e.workers)
          if (h2.cache.key == h.cache.key && h2.cache.digest == h.cache.digest) {
            auto nit = nodes.find(h2.node);
            if (nit != nodes.end() && !nit->second.replica_address.empty()) holders.insert(nit->second.replica_address);
          }
        p.cache_holders.assign(holders.begin(), holders.end());
      }
      pl.members.push_back(p);
    }
    for (auto& sp : e.spares) {
      signals::SparePlacement s;
      if (sp.for_rank >= 0) {
        s.for_rank = (uint32_t)sp.for_rank;
        s.has_for_rank = true;
      }
      s.node = sp.node;
      s.device = sp.device;
      pl.spares.push_back(s);
    }
    for (auto& n : placement_nodes(e))
      if (only_node.empty() || n == only_node) to_node(n, m);
  }

  // ---- spare admission: identity, cordons, pools and the fit of the spare's device -------------
  // Why the standing spare `s` may not take a rank of `e` now ("" when it may). A spare for one
  // rank is held to that rank's device; a spare for any rank to every rank's.
  std::string verdict(const Engine& e, const SpareSeat& s) const {
    auto nit = nodes.find(s.node);
    if (nit != nodes.end() && (nit->second.cordoned || nit->second.drain_by_ms))
      return "node " + s.node + " is cordoned";
    if (!e.fingerprint.empty() && !s.fingerprint.empty() && s.fingerprint != e.fingerprint)
      return "another software identity (build, model, KV format or step configuration)";
    const Device* dev = topo.device(s.node, s.device);
    if (!s.pool.empty()) {
      auto pit = pools.find(s.pool);
      if (pit == pools.end()) return "pool " + s.pool + " no longer exists";
      const PoolSpec& pool = pit->second;
      if (std::find(pool.engines.begin(), pool.engines.end(), e.name) == pool.engines.end())
        return "pool " + s.pool + " no longer holds spares for this engine";
      if (dev != nullptr && !pool.device_class.empty() && dev->cls.find(pool.device_class) == std::string::npos)
        return dev->cls + " is not the pool's class " + pool.device_class;
      if (dev != nullptr && !pool.domain.empty() && dev->domain != pool.domain)
        return "domain " + dev->domain + " is not the pool's " + pool.domain;
    }
    if (dev == nullptr) return "";  // its node reported no devices: nothing to hold it to
    std::vector<uint32_t> ranks;
    if (s.for_rank >= 0) ranks.push_back((uint32_t)s.for_rank);
    else
      for (auto& [r, h] : e.workers) ranks.push_back(r);
    for (uint32_t r : ranks) {
      auto w = e.workers.find(r);
      if (w == e.workers.end()) continue;
      const Device* held = topo.device(w->second.node, w->second.device);
      if (held == nullptr) continue;
      Position pos;
      pos.engine = e.name;
      pos.rank = r;
      pos.cls = held->cls;
      pos.domain = held->domain;
      const Fit f = fit(pos, *dev);
      if (!f.ok) return f.why;
      if (f.same_class) continue;
      char speed[48];
      std::snprintf(speed, sizeof speed, " (speed %.2f)", f.speed);
      if (!policy.spares.allow_mismatched)
        return f.why + speed + ": the policy admits no mismatched spare";
      if (!within_degrade(f, policy.spares.max_degrade_percent))
        return f.why + speed + ": beyond the policy's degrade of " +
               std::to_string(policy.spares.max_degrade_percent) + "%";
    }
    return "";
  }

  // Derive again which standing spares `e` admits; nothing moves while a change is in flight
  // (its spares are spoken for).
  void admit(Engine& e) {
    if (e.in_flight) return;
    std::set<std::pair<std::string, uint32_t>> before;
    for (auto& sp : e.spares) before.insert({sp.node, sp.device});
    std::vector<SpareSeat> next;
    std::map<std::pair<std::string, uint32_t>, std::string> refused;
    for (auto& [key, seat] : e.standing) {
      const std::string why = verdict(e, seat);
      const std::string where = seat.node + ":" + std::to_string(seat.device);
      if (why.empty()) {
        next.push_back(seat);
        if (!before.count(key) && e.refused.count(key))
          event("engine " + e.name + ": spare on " + where + " now qualifies; it stands");
      } else {
        refused[key] = why;
        if (!e.refused.count(key) || e.refused[key] != why) {
          metrics().inc("everserve_spares_refused_total", {{"engine", e.name}});
          event("engine " + e.name + ": spare on " + where + " refused: " + why);
        }
      }
    }
    e.spares = std::move(next);
    e.refused = std::move(refused);
  }

  void readmit_all() {  // after a cordon, a pool write: every engine
    for (auto& [name, e] : engines) {
      const size_t before = e.spares.size();
      admit(e);
      if (e.spares.size() != before) {
        replan(e);
        replicate(e);
      }
    }
    update_gauges(nullptr, true);
  }

  // ---- pools: spare capacity for engines of one shape ------------------------------------------
  void load_pools() {
    std::map<std::string, std::string> all;
    if (!spec || !spec->list("pools/", all)) return;
    for (auto& [key, text] : all) {
      std::string err;
      PoolSpec p;
      if (parse_pool(text, p, err) && !p.name.empty()) pools[p.name] = p;
    }
  }

  // Refuse a spec naming an engine the policy does not know, or engines of different shapes.
  std::string check_pool(const PoolSpec& p) const {
    if (p.name.empty() || p.name.find('/') != std::string::npos || p.name[0] == '.') return "a pool needs a plain name";
    std::string shape;
    for (auto& en : p.engines) {
      auto ep = policy.engines.find(en);
      if (ep == policy.engines.end()) return "the policy names no engine " + en;
      const std::string sh = std::to_string(ep->second.tensor) + "x" + std::to_string(ep->second.pipeline) + "x" +
                             std::to_string(ep->second.data);
      auto e = engines.find(en);
      const std::string fp = e != engines.end() ? e->second.fingerprint : "";
      if (shape.empty()) shape = sh + "|" + fp;
      else if (shape.substr(0, shape.find('|')) != sh ||
               (!fp.empty() && shape.size() > sh.size() + 1 && shape.substr(sh.size() + 1) != fp))
        return "the pool's engines differ in shape (" + en + ")";
    }
    return "";
  }

  struct PoolCount {
    uint32_t standing = 0, warming = 0;
  };
  PoolCount pool_count(const std::string& name) const {
    PoolCount c;
    std::set<std::pair<std::string, uint32_t>> seen;
    for (auto& [en, e] : engines)
      for (auto& [key, seat] : e.standing)
        if (seat.pool == name) seen.insert(key);
    c.standing = (uint32_t)seen.size();
    for (auto& [key, v] : pool_launches)
      if (v.first == name) c.warming++;
    return c;
  }

  // Launch what each pool is short of on free devices of linked, uncordoned nodes.
  void reconcile_pools() {
    if (pools.empty() && pool_launches.empty()) return;
    const uint64_t now = now_ms();
    for (auto it = pool_launches.begin(); it != pool_launches.end();)  // launches that never registered
      it = now - it->second.second > pool_warm_ms ? pool_launches.erase(it) : std::next(it);
    std::set<std::pair<std::string, uint32_t>> busy;
    for (auto& [en, e] : engines) {
      for (auto& [r, h] : e.workers) busy.insert({h.node, h.device});
      for (auto& [key, seat] : e.standing) busy.insert(key);
    }
    for (auto& [key, v] : pool_launches) busy.insert(key);
    for (auto& [name, ep] : policy.engines)
      for (auto& slot : ep.spare_slots) busy.insert({slot.node, slot.device});
    for (auto& [name, pool] : pools) {
      if (pool.command.empty() || pool.engines.empty()) continue;
      const PoolCount c = pool_count(name);
      if (c.standing + c.warming >= pool.wants) continue;
      std::vector<FreeDevice> free;
      for (auto& [node, devs] : topo.all()) {
        auto nit = nodes.find(node);
        if (nit == nodes.end() || !nit->second.linked || nit->second.cordoned || nit->second.drain_by_ms) continue;
        for (auto& d : devs)
          if (!busy.count({node, d.index})) free.push_back({node, d.index, d.cls, d.domain});
      }
      for (auto& [node, device] : place_pool_spares(pool, free, pool.wants - c.standing - c.warming)) {
        coord::CoordToDaemon m;
        m.has_launch_spare = true;
        auto& ls = m.launch_spare;
        ls.pool = name;
        ls.engines = pool.engines;
        ls.engine = pool.engines.size() == 1 ? pool.engines[0] : "";
        ls.device = device;
        ls.command = pool.command;
        ls.env = pool.env;
        to_node(node, m);
        pool_launches[{node, device}] = {name, now};
        busy.insert({node, device});
        for (auto& en : pool.engines) {
          auto eit = engines.find(en);
          if (eit != engines.end()) send_placement(eit->second, node);
        }
        event("pool " + name + ": spare launch asked of " + node + ":" + std::to_string(device));
      }
    }
    for (auto& [name, pool] : pools) {
      const PoolCount c = pool_count(name);
      metrics().set("everserve_pool_spares", {{"pool", name}, {"state", "standing"}}, c.standing);
      metrics().set("everserve_pool_spares", {{"pool", name}, {"state", "warming"}}, c.warming);
      metrics().set("everserve_pool_deficit", {{"pool", name}},
                    pool.wants > c.standing + c.warming ? pool.wants - c.standing - c.warming : 0);
    }
  }

  std::string pool_view_json(const PoolSpec& p) const {
    const PoolCount c = pool_count(p.name);
    const uint32_t have = c.standing + c.warming;
    std::string spares = "[";
    bool first = true;
    std::set<std::pair<std::string, uint32_t>> seen;
    for (auto& [en, e] : engines)
      for (auto& [key, seat] : e.standing)
        if (seat.pool == p.name && seen.insert(key).second) {
          auto r = e.refused.find(key);
          spares += std::string(first ? "" : ",") + "{\"node\":\"" + json_escape(key.first) + "\",\"device\":" +
                    std::to_string(key.second) + ",\"refused\":\"" + json_escape(r == e.refused.end() ? "" : r->second) +
                    "\"}";
          first = false;
        }
    spares += "]";
    return "{\"metadata\":{\"name\":\"" + json_escape(p.name) + "\",\"generation\":" + std::to_string(p.generation) +
           "},\"spec\":" + pool_json(p) + ",\"status\":{\"standing\":" + std::to_string(c.standing) +
           ",\"warming\":" + std::to_string(c.warming) + ",\"short\":" +
           std::to_string(p.wants > have ? p.wants - have : 0) + ",\"spares\":" + spares + "}}";
  }

  // ---- spares the daemons launch ---------------------------------------------------------------
  void launch_spares(const std::string& node) {
    for (auto& [name, ep] : policy.engines) {
      if (ep.launch_command.empty()) continue;
      for (auto& slot : ep.spare_slots) {
        if (slot.node != node) continue;
        coord::CoordToDaemon m;
        m.has_launch_spare = true;
        auto& ls = m.launch_spare;
        ls.engine = name;
        if (slot.rank >= 0) {
          ls.rank = (uint32_t)slot.rank;
          ls.has_rank = true;
        }
        ls.device = slot.device;
        ls.command = ep.launch_command;
        ls.env = ep.launch_env;
        to_node(node, m);
        event("engine " + name + ": spare launch asked of " + node + ":" + std::to_string(slot.device));
      }
    }
  }

  // ---- cover plans -----------------------------------------------------------------------------
  static std::string member_key(const signals::SetMember& m) {
    return m.has_spare ? "R" + std::to_string(m.spare.for_rank) + "@" + m.spare.node + ":" +
                             std::to_string(m.spare.device)
                       : std::to_string(m.rank);
  }

  void replan(Engine& e) {
    if (!policy.cover_enabled || e.down || e.in_flight) return;
    CoverInput in;
    in.engine = e.name;
    in.epoch = e.epoch;
    auto ep = policy.engines.find(e.name);
    in.tp = ep != policy.engines.end() ? ep->second.tensor : std::max<uint32_t>(1, (uint32_t)e.workers.size());
    in.pp = ep != policy.engines.end() ? ep->second.pipeline : 1;
    if (e.workers.size() < (size_t)in.tp * in.pp) return;  // not every rank registered yet
    for (auto& [r, h] : e.workers) in.holders[r] = {h.node, h.device};
    in.spares = e.spares;
    in.max_groups_per_gpu = policy.cover_max_groups_per_gpu;
    auto allows = [&](int32_t o) {
      return std::find(policy.outcomes.begin(), policy.outcomes.end(), o) != policy.outcomes.end();
    };
    in.replace = allows(signals::Outcome_OUTCOME_REPLACE);
    in.shrink = allows(signals::Outcome_OUTCOME_SHRINK) && ep != policy.engines.end() && ep->second.placement_independent;
    std::vector<std::vector<uint32_t>> covers;
    std::vector<Uncovered> uncovered;
    signals::CoverPlan plan = plan_cover(in, &covers, &uncovered);
    e.cover_uncovered = uncovered;
    const std::string sig = plan.serialize();
    if (sig == e.cover_sig) return;
    e.cover_sig = sig;
    plan.generation = ++e.cover_gen;
    e.cover = plan;
    e.cover_covers = covers;
    e.cover_formed.clear();
    e.cover_failed.clear();
    coord::CoordToDaemon m;
    m.has_cover_plan = true;
    m.cover_plan = plan;
    for (auto& node : engine_nodes(e)) to_node(node, m);
    metrics().inc("everserve_cover_plans_total", {{"engine", e.name}});
    event("engine " + e.name + ": cover plan " + std::to_string(plan.generation) + " (" +
          std::to_string(plan.sets.size()) + " sets, " + std::to_string(plan.groups.size()) + " groups)");
    update_cover_gauge(e);
  }

  bool set_covered(const Engine& e, size_t i) const {
    for (uint32_t g : e.cover.sets[i].groups) {
      const auto& grp = e.cover.groups[g];
      auto it = e.cover_formed.find(spans_key(grp.spans));
      if (it == e.cover_formed.end() || it->second.size() < grp.spans.size()) return false;
    }
    return true;
  }

  void update_cover_gauge(const Engine& e) {
    double n = 0;
    for (size_t i = 0; i < e.cover.sets.size(); i++) n += set_covered(e, i);
    metrics().set("everserve_engine_covered_sets", {{"engine", e.name}}, n);
  }

  void on_cover_report(const coord::CoverReport& r) {
    const signals::GroupFormed* f = r.has_formed ? &r.formed : nullptr;
    std::string engine_name;
    uint64_t gen = 0;
    std::vector<signals::SetMember> spans;
    signals::SetMember who;
    if (r.has_formed) engine_name = r.formed.engine, gen = r.formed.generation, spans = r.formed.spans, who = r.formed.member;
    else if (r.has_failed) engine_name = r.failed.engine, gen = r.failed.generation, spans = r.failed.spans, who = r.failed.member;
    else if (r.has_released) engine_name = r.released.engine, gen = r.released.generation, spans = r.released.spans, who = r.released.member;
    else return;
    auto it = engines.find(engine_name);
    if (it == engines.end() || it->second.cover_gen != gen) return;  // a report of an older plan
    Engine& e = it->second;
    const std::string k = spans_key(spans);
    if (f) {
      e.cover_formed[k].insert(member_key(who));
      metrics().observe("everserve_cover_form_seconds", {{"engine", e.name}}, f->seconds);
    } else if (r.has_failed) {
      e.cover_failed[k] = r.failed.error;
      metrics().inc("everserve_cover_failures_total", {{"engine", e.name}});
    } else {
      e.cover_formed[k].erase(member_key(who));
    }
    update_cover_gauge(e);
  }

  // ---- daemon links ----------------------------------------------------------------------------
  static std::string fingerprint_of(const coord::WorkerEvent& ev) {
    if (!ev.has_identity) return "";
    const auto& id = ev.identity;
    return id.engine_commit + "|" + id.torch_version + "|" + id.model + "|" + id.checkpoint_digest + "|" +
           id.model_dtype + "|" + id.kv_format.dtype + ":" + std::to_string(id.kv_format.block_size) + "|" +
           std::to_string(id.layout.tensor) + "x" + std::to_string(id.layout.pipeline) + "|" + id.step.digest;
  }

  void on_worker_event(const std::string& node, const coord::WorkerEvent& ev) {
    Engine& e = engine(ev.engine);
    using K = coord::WorkerEvent_Kind;
    switch (ev.kind) {
      case K::WorkerEvent_Kind_WORKER_REGISTERED: {
        Holder h;
        h.node = node;
        h.device = ev.device;
        h.pid = ev.pid;
        h.host = ev.host;
        if (ev.has_compile_cache) h.cache = ev.compile_cache;
        e.workers[ev.rank] = h;
        if (e.fingerprint.empty()) e.fingerprint = fingerprint_of(ev);
        e.epoch = std::max(e.epoch, ev.epoch);
        if (e.down && e.workers.size() >= std::max<uint32_t>(1, e.world)) {
          e.down = false;
          metrics().set("everserve_engine_down", {{"engine", e.name}}, 0);
        }
        break;
      }
      case K::WorkerEvent_Kind_SPARE_REGISTERED: {
        SpareSeat s;
        s.node = node;
        s.device = ev.device;
        s.for_rank = ev.any_rank ? -1 : (int64_t)ev.rank;
        s.pid = ev.pid;
        s.fingerprint = fingerprint_of(ev);
        auto pl = pool_launches.find({node, ev.device});
        if (pl != pool_launches.end()) s.pool = pl->second.first;
        for (auto& [pname, pool] : pools)  // a pool spare that outlived a restart of this process
          if (s.pool.empty() && ev.any_rank &&
              std::find(pool.engines.begin(), pool.engines.end(), e.name) != pool.engines.end())
            s.pool = pname;
        if (!e.fingerprint.empty() && !s.fingerprint.empty() && s.fingerprint != e.fingerprint)
          metrics().inc("everserve_spares_mismatched_total", {{"engine", e.name}});
        // a daemon announces its processes again on every link: one seat per (node, device)
        e.standing[{node, ev.device}] = s;
        break;
      }
      case K::WorkerEvent_Kind_HEAD_REGISTERED: e.head_nodes.insert(node); break;
      case K::WorkerEvent_Kind_WORKER_DEPARTED: {
        auto it = e.workers.find(ev.rank);
        if (it != e.workers.end() && it->second.node == node && ev.cause != signals::StopCause_STOP_CAUSE_STOPPED)
          report_loss(ev.engine, {ev.rank}, 0, "departed");
        else if (it != e.workers.end() && it->second.node == node)
          e.workers.erase(it);
        break;
      }
      case K::WorkerEvent_Kind_SPARE_DEPARTED:
        e.standing.erase({node, ev.device});
        e.refused.erase({node, ev.device});
        e.spares.erase(std::remove_if(e.spares.begin(), e.spares.end(),
                                      [&](const SpareSeat& s) { return s.node == node && s.device == ev.device; }),
                       e.spares.end());
        break;
      case K::WorkerEvent_Kind_HEAD_DEPARTED: e.head_nodes.erase(node); break;
      default: break;
    }
    if (ev.kind == K::WorkerEvent_Kind_SPARE_REGISTERED) pool_launches.erase({node, ev.device});
    admit(e);
    update_gauges(&e);
    replan(e);
    replicate(e);
    reconcile_pools();
    send_placement(e);
  }

  void from_daemon(Conn& c, const std::string& frame) {
    coord::DaemonToCoord m;
    if (!m.parse(frame)) return;
    std::string node = conn_node.count(c.id) ? conn_node[c.id] : "";
    if (m.has_hello) {
      if (m.hello.protocol != 0 && m.hello.protocol < signals::ProtocolOldest_PROTOCOL_OLDEST) {
        ES_WARN("node %s speaks protocol %u, older than supported", m.hello.node.c_str(), m.hello.protocol);
        loop.close(c.id);
        return;
      }
      if (!c.peer_cn.empty() && c.peer_cn != m.hello.node) {
        ES_WARN("a daemon with the certificate of %s said it is node %s: refused", c.peer_cn.c_str(),
                m.hello.node.c_str());
        metrics().inc("everserve_refused_links_total");
        loop.close(c.id);
        return;
      }
      node = m.hello.node;
      conn_node[c.id] = node;
      Node& n = nodes[node];
      n.name = node;
      n.conn = c.id;
      n.linked = true;
      n.last_seen_ms = now_ms();
      n.heartbeat_ms = m.hello.heartbeat_ms ? m.hello.heartbeat_ms : 500;
      n.replica_address = m.hello.mirror_replica_address;
      std::vector<Device> devs;
      for (auto& d : m.hello.devices) {
        Device dv;
        dv.index = d.index;
        dv.uuid = d.uuid;
        dv.cls = d.class_;
        dv.memory_bytes = d.memory_bytes;
        dv.domain = d.domain;
        devs.push_back(dv);
      }
      topo.set_node(node, std::move(devs));
      for (auto& st : m.hello.engines) {
        Engine& e = engine(st.engine);
        e.epoch = std::max(e.epoch, st.epoch);
      }
      event("node " + node + " linked (" + std::to_string(m.hello.devices.size()) + " device(s))");
      // this node's devices change the fit of spares on it and of positions held on it
      for (auto& [ename, en] : engines)
        if (needs_placement(en, node)) {
          admit(en);
          send_placement(en, node);  // what this node's processes need
        }
      launch_spares(node);
      reconcile_pools();
      loop.every(200, [this] {
        for (auto& [name, en] : engines) try_resume(en);
      }, false);
      return;
    }
    if (node.empty()) return;  // nothing before a hello
    nodes[node].last_seen_ms = now_ms();
    if (m.has_heartbeat) return;
    if (m.has_bye) {
      nodes[node].linked = false;
      return;
    }
    if (m.has_worker_event) on_worker_event(node, m.worker_event);
    else if (m.has_lost_report) {
      std::vector<uint32_t> ranks(m.lost_report.lost.ranks.begin(), m.lost_report.lost.ranks.end());
      report_loss(m.lost_report.engine, ranks, m.lost_report.lost.epoch,
                  m.lost_report.lost.reason == signals::Reason_REASON_NOTICE ? "notice" : "fault",
                  m.lost_report.lost.reason == signals::Reason_REASON_NOTICE);
    } else if (m.has_notice_report) {
      report_loss(m.notice_report.engine, {m.notice_report.notice.rank}, 0, "notice", true);
    } else if (m.has_delivered) {
      delivered(node, m.delivered);
    } else if (m.has_join_report) {
      // joins are opaque bytes between the head and the ranks: relay to every node of the engine
      coord::CoordToDaemon out;
      out.has_forward_join = true;
      out.forward_join.engine = m.join_report.engine;
      out.forward_join.join = m.join_report.join;
      out.forward_join.has_join = true;
      out.forward_join.to_clients = !m.join_report.from_client;
      auto it = engines.find(m.join_report.engine);
      if (it != engines.end())
        for (auto& n : engine_nodes(it->second)) to_node(n, out);
    } else if (m.has_role_asked) {
      coord::CoordToDaemon out;
      out.has_role_answer = true;
      out.role_answer.request_id = m.role_asked.request_id;
      out.role_answer.engine = m.role_asked.engine;
      out.role_answer.rank = m.role_asked.rank;
      Engine& e = engine(m.role_asked.engine);
      out.role_answer.epoch = e.epoch;
      out.role_answer.role = e.workers.count(m.role_asked.rank) ? signals::Role_ROLE_SPARE : signals::Role_ROLE_WORKER;
      to_node(node, out);
    } else if (m.has_node_notice) {
      drain(node, m.node_notice.deadline_ms, "node notice: " + m.node_notice.source);
    } else if (m.has_stacks_sent) {
      auto& v = stacks[m.stacks_sent.request_id];
      v.emplace_back(node + ":" + std::to_string(m.stacks_sent.pid),
                     m.stacks_sent.answered ? m.stacks_sent.text : "(no answer: " + m.stacks_sent.error + ")");
      while (stacks.size() > 64) stacks.erase(stacks.begin());
    } else if (m.has_release_leaked) {
      // a process could not release a refused group within its bound: it holds what a stuck
      // communicator holds, so it is retired by notice (it finishes its step; a spare takes the
      // rank at the boundary) when a spare can take its rank, and counted either way
      const auto& lk = m.release_leaked.leak;
      metrics().inc("everserve_releases_leaked_total", {{"engine", lk.engine}});
      event("engine " + lk.engine + ": rank " + std::to_string(lk.rank) + " on " + node + " leaked a release (" +
            lk.release + ", " + std::to_string(lk.run_ms) + " ms)");
      auto it = engines.find(lk.engine);
      if (it != engines.end()) {
        Engine& e = it->second;
        auto w = e.workers.find(lk.rank);
        const bool spare = std::any_of(e.spares.begin(), e.spares.end(), [&](const SpareSeat& s) {
          return s.for_rank < 0 || s.for_rank == (int64_t)lk.rank;
        });
        if (w != e.workers.end() && w->second.node == node && spare)
          report_loss(lk.engine, {lk.rank}, 0, "release leaked", true);
      }
    } else if (m.has_cover_report) {
      on_cover_report(m.cover_report);
    } else if (m.has_replay_ask || m.has_replay_offer) {
      coord::CoordToDaemon out;
      std::string eng;
      if (m.has_replay_ask) {
        out.has_replay_ask = true;
        out.replay_ask = m.replay_ask;
        eng = m.replay_ask.engine;
        // a process starting for the engine on this node (a spare): it will want the placement
        Engine& le = engine(eng);
        if (le.listeners.insert(node).second) send_placement(le, node);
      } else {
        // an offer goes back to the node of the process that asked
        out.has_replay_offer = true;
        out.replay_offer = m.replay_offer;
        to_node(m.replay_offer.to.node, out);
        return;
      }
      auto it = engines.find(eng);
      if (it != engines.end())
        for (auto& n : engine_nodes(it->second)) to_node(n, out);
    }
  }

  void link_closed(Conn& c) {
    auto it = conn_node.find(c.id);
    if (it == conn_node.end()) return;
    const std::string node = it->second;
    conn_node.erase(it);
    Node& n = nodes[node];
    if (n.conn != c.id) return;
    n.linked = false;
    node_lost(node, "link ended");
  }

  void node_lost(const std::string& node, const std::string& why) {
    event("node " + node + " lost: " + why);
    for (auto& [name, e] : engines) {
      std::vector<uint32_t> ranks;
      for (auto& [r, h] : e.workers)
        if (h.node == node) ranks.push_back(r);
      e.spares.erase(std::remove_if(e.spares.begin(), e.spares.end(), [&](const SpareSeat& s) { return s.node == node; }),
                     e.spares.end());
      for (auto it = e.standing.begin(); it != e.standing.end();)
        it = it->first.first == node ? e.standing.erase(it) : std::next(it);
      for (auto it = e.refused.begin(); it != e.refused.end();)
        it = it->first.first == node ? e.refused.erase(it) : std::next(it);
      if (e.in_flight && e.in_flight->waiting.count(node)) abandon(e, "node " + node + " lost during the change");
      if (!ranks.empty()) report_loss(name, ranks, 0, "node lost");
    }
    for (auto it = pool_launches.begin(); it != pool_launches.end();)
      it = it->first.first == node ? pool_launches.erase(it) : std::next(it);
    topo.remove_node(node);
    update_gauges(nullptr, true);
    reconcile_pools();
  }

  void check_heartbeats() {
    const uint64_t now = now_ms();
    for (auto& [name, n] : nodes) {
      if (n.linked && now - n.last_seen_ms > (uint64_t)n.heartbeat_ms * loss_misses) {
        n.linked = false;
        loop.close(n.conn);
        node_lost(name, std::to_string(loss_misses) + " heartbeats missed");
      }
    }
  }

  void drain(const std::string& node, int64_t deadline_ms, const std::string& why) {
    Node& n = nodes[node];
    n.name = node;
    n.drain_by_ms = deadline_ms ? deadline_ms : (int64_t)now_ms();
    write_node(n);
    event("node " + node + " draining (" + why + ")");
    for (auto& [name, e] : engines) {
      std::vector<uint32_t> ranks;
      for (auto& [r, h] : e.workers)
        if (h.node == node) ranks.push_back(r);
      if (!ranks.empty()) report_loss(name, ranks, 0, "notice", true);
    }
  }

  // ---- readiness -------------------------------------------------------------------------------
  // Whether `node` can be drained now without an engine going down: every rank it holds has an
  // admitted spare on another node (distinct spares; a spare for one rank only takes that rank).
  std::string reclaim_blocker(const std::string& node) const {
    for (auto& [name, e] : engines) {
      std::vector<uint32_t> ranks;
      for (auto& [r, h] : e.workers)
        if (h.node == node) ranks.push_back(r);
      if (ranks.empty()) continue;
      std::vector<SpareSeat> seats;
      for (auto& sp : e.spares)
        if (sp.node != node) seats.push_back(sp);
      std::vector<bool> used(seats.size(), false);
      for (uint32_t r : ranks) {
        int pick = -1;
        for (size_t i = 0; i < seats.size() && pick < 0; i++)
          if (!used[i] && seats[i].for_rank == (int64_t)r) pick = (int)i;
        for (size_t i = 0; i < seats.size() && pick < 0; i++)
          if (!used[i] && seats[i].for_rank < 0) pick = (int)i;
        if (pick < 0) return "engine " + name + " rank " + std::to_string(r) + " has no spare on another node";
        used[(size_t)pick] = true;
      }
    }
    return "";
  }

  // The pause a loss is expected to cost now: the median of the engine's recent changes (null
  // before its first).
  std::string expected_pause_json(const Engine& e) const {
    if (e.pauses_ms.empty()) return "null";
    std::vector<double> v(e.pauses_ms.begin(), e.pauses_ms.end());
    std::sort(v.begin(), v.end());
    char buf[32];
    std::snprintf(buf, sizeof buf, "%.3f", v[v.size() / 2]);
    return buf;
  }

  // ---- operator API ----------------------------------------------------------------------------
  std::string engine_json(const Engine& e) {
    std::string w = "[";
    bool first = true;
    for (auto& [r, h] : e.workers) {
      w += std::string(first ? "" : ",") + "{\"rank\":" + std::to_string(r) + ",\"node\":\"" + json_escape(h.node) +
           "\",\"device\":" + std::to_string(h.device) + "}";
      first = false;
    }
    w += "]";
    std::string s = "[";
    first = true;
    for (auto& sp : e.spares) {
      s += std::string(first ? "" : ",") + "{\"node\":\"" + json_escape(sp.node) + "\",\"device\":" +
           std::to_string(sp.device) + ",\"forRank\":" + std::to_string(sp.for_rank) + ",\"pool\":\"" +
           json_escape(sp.pool) + "\"}";
      first = false;
    }
    s += "]";
    std::string refused = "[";
    first = true;
    for (auto& [key, why] : e.refused) {
      const SpareSeat& seat = e.standing.at(key);
      refused += std::string(first ? "" : ",") + "{\"node\":\"" + json_escape(key.first) + "\",\"device\":" +
                 std::to_string(key.second) + ",\"forRank\":" + std::to_string(seat.for_rank) + ",\"why\":\"" +
                 json_escape(why) + "\"}";
      first = false;
    }
    refused += "]";
    // conditions, as an operator reads them
    const uint32_t world = e.world ? e.world : (uint32_t)e.workers.size();
    size_t covered = 0, replacements = 0;
    for (size_t i = 0; i < e.cover.sets.size(); i++) {
      if (i < e.cover_covers.size() && !e.cover_covers[i].empty()) {
        replacements++;
        covered += set_covered(e, i);
      }
    }
    auto cond = [](const std::string& type, bool status, const std::string& reason) {
      return "{\"type\":\"" + type + "\",\"status\":\"" + (status ? "True" : "False") + "\",\"reason\":\"" +
             json_escape(reason) + "\"}";
    };
    const bool ready = !e.down && !e.in_flight && e.workers.size() >= world && world > 0;
    std::string conds = "[" +
        cond("Ready", ready, e.down ? "a change was abandoned" : e.in_flight ? "a change is in flight"
                                   : e.workers.size() < world ? "ranks missing" : "serving") + "," +
        cond("Progressing", (bool)e.in_flight, e.in_flight ? "change to epoch " + std::to_string(e.in_flight->change.epoch) : "") + "," +
        cond("Degraded", e.down || e.spares.empty(), e.down ? "engine down" : e.spares.empty() ? "no standing spare" : "") + "," +
        cond("Covered", replacements > 0 && covered == replacements,
             std::to_string(covered) + " of " + std::to_string(replacements) + " replacement sets formed") + "]";
    for (auto& [type, st] : std::vector<std::pair<std::string, bool>>{
             {"Ready", ready}, {"Progressing", (bool)e.in_flight}, {"Degraded", e.down || e.spares.empty()},
             {"Covered", replacements > 0 && covered == replacements}})
      metrics().set("everserve_engine_condition", {{"engine", e.name}, {"type", type}}, st ? 1 : 0);
    std::string cov = "{\"generation\":" + std::to_string(e.cover_gen) + ",\"sets\":[";
    for (size_t i = 0; i < e.cover.sets.size(); i++) {
      std::string ranks = "[";
      if (i < e.cover_covers.size())
        for (size_t k = 0; k < e.cover_covers[i].size(); k++)
          ranks += (k ? "," : "") + std::to_string(e.cover_covers[i][k]);
      cov += std::string(i ? "," : "") + "{\"purpose\":\"" + json_escape(e.cover.sets[i].purpose) + "\",\"covers\":" +
             ranks + "],\"covered\":" + (set_covered(e, i) ? "true" : "false") + "}";
    }
    cov += "],\"uncovered\":[";
    for (size_t i = 0; i < e.cover_uncovered.size(); i++) {
      const auto& u = e.cover_uncovered[i];
      std::string ranks = "[";
      for (size_t k = 0; k < u.lost.size(); k++) ranks += (k ? "," : "") + std::to_string(u.lost[k]);
      cov += std::string(i ? "," : "") + "{\"lost\":" + ranks + "],\"why\":\"" + json_escape(u.why) + "\"}";
    }
    cov += "]}";
    return "{\"metadata\":{\"name\":\"" + json_escape(e.name) + "\"},\"status\":{\"epoch\":" + std::to_string(e.epoch) +
           ",\"worldSize\":" + std::to_string(e.world) + ",\"down\":" + (e.down ? "true" : "false") +
           ",\"changing\":" + (e.in_flight ? "true" : "false") + ",\"workers\":" + w + ",\"spares\":" + s + ",\"refusedSpares\":" + refused + ",\"expectedPauseMs\":" +
           expected_pause_json(e) + ",\"cover\":" + cov + ",\"conditions\":" + conds + "}}";
  }

  bool api(const HttpRequest& req, HttpResponse& resp) {
    resp.content_type = "application/json";
    const std::string path = req.path.substr(0, req.path.find('?'));
    if (req.method == "GET" && path == "/v1/engines") {
      std::string o = "{\"items\":[";
      bool first = true;
      for (auto& [n, e] : engines) {
        o += (first ? "" : ",") + engine_json(e);
        first = false;
      }
      resp.body = o + "]}";
      return true;
    }
    if (req.method == "GET" && path.rfind("/v1/engines/", 0) == 0 && path.find('/', 12) == std::string::npos) {
      const std::string name = path.substr(12);
      auto it = engines.find(name);
      if (it == engines.end()) return false;
      resp.body = engine_json(it->second);
      return true;
    }
    if (req.method == "GET" && path == "/v1/nodes") {
      std::string o = "{\"items\":[";
      bool first = true;
      for (auto& [name, n] : nodes) {
        std::string devs = "[";
        if (const auto* ds = topo.node(name))
          for (size_t i = 0; i < ds->size(); i++) {
            const Device& d = (*ds)[i];
            devs += std::string(i ? "," : "") + "{\"index\":" + std::to_string(d.index) + ",\"uuid\":\"" +
                    json_escape(d.uuid) + "\",\"class\":\"" + json_escape(d.cls) + "\",\"memoryBytes\":" +
                    std::to_string(d.memory_bytes) + ",\"domain\":\"" + json_escape(d.domain) + "\"}";
          }
        devs += "]";
        o += std::string(first ? "" : ",") + "{\"metadata\":{\"name\":\"" + json_escape(name) + "\"},\"spec\":{\"unschedulable\":" +
             (n.cordoned ? "true" : "false") + ",\"drainByMs\":" + std::to_string(n.drain_by_ms) + "},\"status\":{\"linked\":" +
             (n.linked ? "true" : "false") + ",\"domain\":\"" + json_escape(topo.domain_of(name)) + "\",\"devices\":" + devs +
             ",\"reclaimable\":" + (reclaim_blocker(name).empty() ? "true" : "false") + ",\"reclaimBlocker\":\"" +
             json_escape(reclaim_blocker(name)) + "\"}}";
        first = false;
      }
      resp.body = o + "]}";
      return true;
    }
    if (req.method == "PUT" && path.rfind("/v1/nodes/", 0) == 0) {
      std::string rest = path.substr(10);
      const auto slash = rest.find('/');
      const std::string node = rest.substr(0, slash), verb = slash == std::string::npos ? "" : rest.substr(slash + 1);
      Node& n = nodes[node];
      n.name = node;
      if (verb == "cordon") n.cordoned = true;
      else if (verb == "uncordon") n.cordoned = false;
      else if (verb == "drain") {
        n.cordoned = true;
        drain(node, 0, "operator");
      } else if (verb == "undrain") n.drain_by_ms = 0;
      else return false;
      write_node(n);
      readmit_all();
      reconcile_pools();
      resp.body = "{\"node\":\"" + json_escape(node) + "\",\"done\":\"" + verb + "\"}";
      return true;
    }
    if (req.method == "GET" && path.rfind("/v1/engines/", 0) == 0 && path.size() > 7 &&
        path.compare(path.size() - 7, 7, "/events") == 0) {
      const std::string name = path.substr(12, path.size() - 12 - 7);
      std::string o = "{\"engine\":\"" + json_escape(name) + "\",\"events\":[";
      bool first = true;
      for (auto& ev : events)
        if (ev.engine == name) {
          o += std::string(first ? "" : ",") + "{\"seq\":" + std::to_string(ev.seq) + ",\"atMs\":" +
               std::to_string(ev.at_ms) + ",\"text\":\"" + json_escape(ev.text) + "\"}";
          first = false;
        }
      resp.body = o + "]}";
      return true;
    }
    if (req.method == "GET" && path.rfind("/v1/stacks/", 0) == 0) {
      const uint64_t id = std::stoull(path.substr(11));
      auto it = stacks.find(id);
      std::string o = "{\"request\":" + std::to_string(id) + ",\"processes\":[";
      bool first = true;
      if (it != stacks.end())
        for (auto& [who, text] : it->second) {
          o += std::string(first ? "" : ",") + "{\"process\":\"" + json_escape(who) + "\",\"stacks\":\"" +
               json_escape(text) + "\"}";
          first = false;
        }
      resp.body = o + "]}";
      return true;
    }
    if (req.method == "GET" && path == "/v1/watch") {
      uint64_t since = 0;
      const auto q = req.path.find("since=");
      if (q != std::string::npos) since = std::stoull(req.path.substr(q + 6));
      std::string o = "{\"events\":[";
      bool first = true;
      for (auto& ev : events)
        if (ev.seq > since) {
          o += std::string(first ? "" : ",") + "{\"seq\":" + std::to_string(ev.seq) + ",\"atMs\":" + std::to_string(ev.at_ms) +
               ",\"text\":\"" + json_escape(ev.text) + "\"}";
          first = false;
        }
      resp.body = o + "]}";
      return true;
    }
    if (req.method == "POST" && path.rfind("/v1/engines/", 0) == 0 && path.size() > 7 &&
        path.compare(path.size() - 7, 7, "/stacks") == 0) {
      const std::string name = path.substr(12, path.size() - 12 - 7);
      auto it = engines.find(name);
      if (it == engines.end()) return false;
      coord::CoordToDaemon m;
      m.has_stacks = true;
      m.stacks.request_id = next_request++;
      m.stacks.engine = name;
      for (auto& node : engine_nodes(it->second)) to_node(node, m);
      resp.body = "{\"requested\":" + std::to_string(m.stacks.request_id) + "}";
      return true;
    }
    if (path == "/v1/pools" && req.method == "GET") {
      std::string o = "{\"items\":[";
      bool first = true;
      for (auto& [name, p] : pools) {
        o += (first ? "" : ",") + pool_view_json(p);
        first = false;
      }
      resp.body = o + "]}";
      return true;
    }
    if (path.rfind("/v1/pools/", 0) == 0) {
      const std::string name = path.substr(10);
      auto it = pools.find(name);
      if (req.method == "GET") {
        if (it == pools.end()) return false;
        resp.body = pool_view_json(it->second);
        return true;
      }
      if (req.method == "DELETE") {
        if (it == pools.end()) return false;
        pools.erase(it);
        if (spec) spec->remove("pools/" + name + ".json");
        metrics().inc("everserve_spec_writes_total", {{"kind", "pool"}, {"verdict", "deleted"}});
        event("pool " + name + " deleted");
        readmit_all();
        resp.body = "{\"deleted\":\"" + json_escape(name) + "\"}";
        return true;
      }
      if (req.method == "PUT") {
        PoolSpec p;
        std::string err;
        if (!parse_pool(req.body, p, err)) {
          resp.status = 400;
          resp.body = "{\"error\":\"" + json_escape(err) + "\"}";
          return true;
        }
        p.name = name;
        const uint64_t held = it == pools.end() ? 0 : it->second.generation;
        const auto q = req.path.find("generation=");
        if (q != std::string::npos && std::stoull(req.path.substr(q + 11)) != held) {
          resp.status = 409;
          resp.body = "{\"error\":\"" + json_escape(name) + ": written against generation " + req.path.substr(q + 11) +
                      ", and generation " + std::to_string(held) + " is held\"}";
          return true;
        }
        const std::string why = check_pool(p);
        if (!why.empty()) {
          resp.status = 400;
          resp.body = "{\"error\":\"" + json_escape(why) + "\"}";
          metrics().inc("everserve_spec_writes_total", {{"kind", "pool"}, {"verdict", "refused"}});
          return true;
        }
        p.generation = held + 1;
        if (spec) {
          if (!spec->put("pools/" + name + ".json", pool_json(p))) {
            resp.status = 500;
            resp.body = "{\"error\":\"the spec store refused the write\"}";
            return true;
          }
        }
        pools[name] = p;
        metrics().inc("everserve_spec_writes_total", {{"kind", "pool"}, {"verdict", "written"}});
        event("pool " + name + " written (generation " + std::to_string(p.generation) + ", wants " +
              std::to_string(p.wants) + ")");
        readmit_all();
        reconcile_pools();
        resp.body = pool_view_json(p);
        return true;
      }
      return false;
    }
    if (req.method == "GET" && path == "/v1/openapi") {
      resp.body =
          "{\"openapi\":\"3.0.0\",\"info\":{\"title\":\"everserve coordinator\",\"version\":\"1\"},\"paths\":{"
          "\"/v1/engines\":{\"get\":{}},\"/v1/engines/{name}\":{\"get\":{}},\"/v1/engines/{name}/events\":{\"get\":{}},\"/v1/engines/{name}/stacks\":{\"post\":{}},\"/v1/stacks/{request}\":{\"get\":{}},"
          "\"/v1/nodes\":{\"get\":{}},\"/v1/nodes/{name}/{cordon|uncordon|drain|undrain}\":{\"put\":{}},"
          "\"/v1/pools\":{\"get\":{}},\"/v1/pools/{name}\":{\"get\":{},\"put\":{},\"delete\":{}},"
          "\"/v1/watch\":{\"get\":{}}}}";
      return true;
    }
    return false;
  }
};

}  // namespace

int main(int argc, char** argv) {
  {
    std::string terr;
    if (!es::tls::configure_from_env(&terr)) {
      fprintf(stderr, "TLS: %s\n", terr.c_str());
      return 2;
    }
  }
  log_init("coord");
  signal(SIGPIPE, SIG_IGN);
  Coordinator co;
  std::string listen = env_or("EVERSERVE_LISTEN", "unix:/tmp/everserve-coord.sock");
  std::string policy_path = env_or("EVERSERVE_POLICY", "");
  co.spec_dir = env_or("EVERSERVE_SPEC_STORE", "");
  std::string lease = env_or("EVERSERVE_LEASE", "");
  std::string api_addr = env_or("EVERSERVE_API_ADDR", "");
  std::string metrics_addr = env_or("EVERSERVE_METRICS_ADDR", "");
  co.loss_misses = (uint32_t)std::stoul(env_or("EVERSERVE_NODE_LOSS_MISSES", "3"));
  co.fold_ms = std::stoull(env_or("EVERSERVE_FOLD_MS", "3"));
  std::string lease_holder = env_or("EVERSERVE_LEASE_HOLDER", "");
  std::string enroll_addr = env_or("EVERSERVE_ENROLL_ADDR", "");
  std::string enroll_ca_dir = env_or("EVERSERVE_ENROLL_CA_DIR", env_or("EVERSERVE_TLS_DIR", ""));
  int enroll_hours = std::stoi(env_or("EVERSERVE_ENROLL_HOURS", "12"));
  std::string api_auth = env_or("EVERSERVE_API_AUTH", "cert");
  std::string api_namespace = env_or("EVERSERVE_API_NAMESPACE", "");
  uint32_t lease_duration_s = (uint32_t)std::stoul(env_or("EVERSERVE_LEASE_DURATION_S", "15"));
  for (int i = 1; i + 1 < argc; i += 2) {
    const std::string k = argv[i], v = argv[i + 1];
    if (k == "--listen") listen = v;
    else if (k == "--policy") policy_path = v;
    else if (k == "--spec-store") co.spec_dir = v;
    else if (k == "--lease") lease = v;
    else if (k == "--api-addr") api_addr = v;
    else if (k == "--metrics-addr") metrics_addr = v;
    else if (k == "--node-loss-misses") co.loss_misses = (uint32_t)std::stoul(v);
    else if (k == "--delivery-timeout-ms") co.delivery_timeout_ms = std::stoull(v);
    else if (k == "--fold-ms") co.fold_ms = std::stoull(v);
    else if (k == "--lease-holder") lease_holder = v;
    else if (k == "--enroll-addr") enroll_addr = v;
    else if (k == "--enroll-ca-dir") enroll_ca_dir = v;
    else if (k == "--enroll-hours") enroll_hours = std::stoi(v);
    else if (k == "--api-auth") api_auth = v;
    else if (k == "--api-namespace") api_namespace = v;
    else if (k == "--lease-duration-s") lease_duration_s = (uint32_t)std::stoul(v);
    else {
      fprintf(stderr, "unknown flag %s\n", k.c_str());
      return 2;
    }
  }
  std::string err;
  if (!policy_path.empty()) {
    std::string text;
    if (!read_file(policy_path, text) || !parse_policy(text, co.policy, err)) {
      ES_ERROR("policy %s: %s", policy_path.c_str(), err.c_str());
      return 1;
    }
  } else {
    co.policy.outcomes = {signals::Outcome_OUTCOME_REPLACE};
  }
  std::unique_ptr<Lease> held;
  if (!lease.empty()) {
    if (lease_holder.empty()) {
      char host[256] = {0};
      gethostname(host, sizeof(host) - 1);
      lease_holder = std::string(host) + ":" + std::to_string(getpid());
    }
    held = make_lease(lease, lease_holder, lease_duration_s);
    if (!held->acquire(co.term, err)) {
      ES_ERROR("lease %s: %s", lease.c_str(), err.c_str());
      return 1;
    }
    ES_INFO("lease %s held by %s, term %llu", lease.c_str(), lease_holder.c_str(), (unsigned long long)co.term);
    if (const uint64_t every = held->renew_every_ms()) {
      // renewed off the loop; a holder that lost its lease stops at once (a successor may write)
      std::thread([every, &held, lease] {
        for (;;) {
          std::this_thread::sleep_for(std::chrono::milliseconds(every));
          std::string e;
          if (!held->renew(e)) {
            ES_ERROR("lease %s lost: %s; exiting", lease.c_str(), e.c_str());
            _exit(3);
          }
        }
      }).detach();
    }
  }
  co.exit_after_log = env_or("EVERSERVE_COORD_EXIT_AFTER_LOG", "") == "1";
  co.spec = make_spec_store(co.spec_dir);
  co.load_spec();
  co.load_pools();
  co.load_nodes();
  metrics().describe("everserve_changes_total", "Membership changes by engine, cause, outcome and verdict", "counter");
  metrics().describe("everserve_change_seconds", "From the first loss report to the commit", "histogram");
  metrics().describe("everserve_change_decision_seconds", "Time to choose an outcome", "histogram");
  metrics().describe("everserve_changes_in_flight", "1 while an engine's change is in flight", "gauge");
  metrics().describe("everserve_daemons_connected", "Linked node daemons", "gauge");
  metrics().describe("everserve_workers_registered", "Workers of every engine", "gauge");
  metrics().describe("everserve_spares", "Spares by engine and state", "gauge");
  metrics().describe("everserve_engine_down", "1 for an engine whose change was abandoned", "gauge");
  metrics().describe("everserve_spec_writes_total", "Writes to the spec store", "counter");
  metrics().describe("everserve_cover_plans_total", "Cover plans sent per engine", "counter");
  metrics().describe("everserve_engine_condition", "1 when an engine condition (Ready, Progressing, Degraded, Covered) holds", "gauge");
  metrics().describe("everserve_engine_covered_sets", "Planned member sets whose groups every member formed", "gauge");
  metrics().describe("everserve_cover_form_seconds", "Time a member took to form a planned group", "histogram");
  metrics().describe("everserve_cover_failures_total", "Planned groups a member failed to form", "counter");
  metrics().describe("everserve_fenced_total", "Reports dropped as older than the engine's epoch", "counter");
  metrics().describe("everserve_spares_refused_total", "Spares refused admission (identity, cordon, pool, device fit)", "counter");
  metrics().describe("everserve_api_refusals_total", "Operator API requests refused by the token gate, by code", "counter");
  metrics().describe("everserve_releases_leaked_total", "Refused groups a process could not release within its bound", "counter");
  metrics().describe("everserve_enrollments_total", "Node certificate requests by verdict (issued, refused)", "counter");
  metrics().describe("everserve_pool_spares", "Spares of each pool by state (standing, warming)", "gauge");
  metrics().describe("everserve_pool_deficit", "Spares a pool wants beyond those standing or warming", "gauge");
  metrics().describe("everserve_unheard_ranks_lost_total", "Loss reports naming ranks the coordinator does not hold", "counter");
  Address a;
  if (!Address::parse(listen, a) || !co.loop.listen(a, [&](Conn& c) {
        c.on_frame = [&](Conn& cc, const std::string& f) { co.from_daemon(cc, f); };
        c.on_close = [&](Conn& cc) { co.link_closed(cc); };
      }, &err)) {
    ES_ERROR("listen %s: %s", listen.c_str(), err.c_str());
    return 1;
  }
  std::unique_ptr<KubeGate> gate;
  HttpOptions api_opt;
  if (api_auth == "kube") {
    // bearer tokens reviewed by the Kubernetes API server instead of client certificates
    if (api_namespace.empty() && !read_file("/var/run/secrets/kubernetes.io/serviceaccount/namespace", api_namespace))
      api_namespace = "default";
    gate = std::make_unique<KubeGate>(KubeClient::from_env(), api_namespace);
    KubeGate* g = gate.get();
    api_opt.client_cert = false;
    api_opt.gate = [g](const HttpRequest& r, HttpResponse& s) { return g->admit(r, s); };
  } else if (api_auth != "cert") {
    ES_ERROR("--api-auth is cert or kube");
    return 2;
  }
  if (!api_addr.empty() &&
      !serve_http(co.loop, api_addr, [&](const HttpRequest& r, HttpResponse& s) { return co.api(r, s); }, &err,
                  api_opt)) {
    ES_ERROR("api %s: %s", api_addr.c_str(), err.c_str());
    return 1;
  }
  std::unique_ptr<Issuer> issuer;
  if (!enroll_addr.empty()) {
    if (enroll_ca_dir.empty()) {
      ES_ERROR("--enroll-addr needs the CA's directory (--enroll-ca-dir or EVERSERVE_TLS_DIR)");
      return 1;
    }
    issuer = std::make_unique<Issuer>(KubeClient::from_env(), enroll_ca_dir, enroll_hours);
    HttpOptions open;
    open.client_cert = false;     // the node has no certificate yet: the token proves it
    open.route_on_loop = false;   // the review waits on the API server
    Issuer* is = issuer.get();
    if (!serve_http(co.loop, enroll_addr, [is](const HttpRequest& r, HttpResponse& s) { return is->route(r, s); },
                    &err, open)) {
      ES_ERROR("enroll %s: %s", enroll_addr.c_str(), err.c_str());
      return 1;
    }
  }
  if (!metrics_addr.empty() && metrics_addr != api_addr && !serve_http(co.loop, metrics_addr, nullptr, &err)) {
    ES_ERROR("metrics %s: %s", metrics_addr.c_str(), err.c_str());
    return 1;
  }
  co.loop.every(tls::reload_period_ms(), [] {  // renewed certificates, taken without a restart
    std::string terr;
    if (!tls::reload_if_changed(&terr)) ES_WARN("TLS reload: %s", terr.c_str());
  });
  co.loop.every(100, [&] { co.check_heartbeats(); });
  co.loop.every(1000, [&] {
    co.reconcile_pools();
    co.fleet_gauges();
  });
  ES_INFO("coordinator term %llu listening on %s", (unsigned long long)co.term, listen.c_str());
  co.loop.run();
  return 0;
}
