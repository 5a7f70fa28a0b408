// everserve-node: the per-node daemon.
//
//   everserve-node --node NAME --socket unix:/run/everserve/node.sock --coordinator ADDR
//                  [--heartbeat-ms 500] [--metrics-addr host:port] [--ack-timeout-ms 120000]
//                  [--mirror-socket ADDR] [--discovery-dir DIR] [--devices-from nvidia-smi|none|PROGRAM]
//                  [--domain NAME] [--cache-wait-ms 600000] [--enroll URL --tls-dir DIR]
// Flags also read EVERSERVE_NODE, EVERSERVE_SOCKET, EVERSERVE_COORDINATOR, EVERSERVE_HEARTBEAT_MS,
// EVERSERVE_METRICS_ADDR, EVERSERVE_MIRROR_SOCKET, EVERSERVE_DISCOVERY_DIR, EVERSERVE_DEVICES_FROM,
// EVERSERVE_DOMAIN.
//
// The node's GPUs (index, UUID, product name, memory) are listed once at start by
// `nvidia-smi --query-gpu=...` (or another program answering the same query) and sent in every
// hello; `--domain` names the NVLink domain they reach at full speed (default: the node).
// A process's CacheWanted is answered once the coordinator's placement names its rank's
// compile-cache pair: the node's store fetches the set from the stores holding it (CacheFetch),
// then CacheReady (or CacheRefused with the reason; no pair within --cache-wait-ms).
//
// Processes of the node (workers, spares, heads, clients) connect to the Unix socket and speak
// signals.proto. The daemon:
//   * records each Register and reports it to the coordinator (WorkerEvent); a connection that
//     ends without a Goodbye is reported as departed (STOP_CAUSE_LOST);
//   * forwards RankLost / Notice / Join / cover reports / replay offers up;
//   * delivers a coordinator's Change to the named ranks and spares, collects their Acks (bounded
//     by the ack timeout) and answers Delivered; relays MembershipCommitted / Abandon / joins /
//     cover plans / replay messages down to the engine's processes;
//   * links to the coordinator with a hello and heartbeats, reconnecting with jittered backoff;
//     reports made while unlinked are held and sent on the next link. Messages from an older
//     coordinator term than the highest seen are ignored (fencing).
#include <signal.h>
#include <sys/socket.h>
#include <sys/wait.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cstring>
#include <deque>
#include <map>
#include <random>
#include <set>
#include <thread>

#include "enroll.h"
#include "everserve_pb.h"
#include "frame.h"
#include "kube.h"
#include "net.h"
#include "notice.h"
#include "telemetry.h"
#include "tls.h"
#include "util.h"

using namespace es;

namespace {

struct Proc {
  uint64_t conn = 0;
  std::string engine;
  uint32_t rank = 0;
  int32_t role = signals::Role_ROLE_UNDECIDED;
  bool any_rank = false;
  uint32_t pid = 0;
  uint32_t device = 0;
  bool registered = false;
  bool said_goodbye = false;
  int32_t goodbye_cause = 0;   // the cause its Goodbye named (STOPPED when it named none)
  bool reported_gone = false;  // its departure was reported (by the process watcher or the close)
  int os_pid = 0;              // the peer's pid in this daemon's pid namespace (SO_PEERCRED), 0 unknown
  signals::Register reg;
};

// A process is leaving once the kernel has started its exit (PF_EXITING), it is a zombie or gone,
// or SIGKILL is pending: that is seen within the poll period, well before its sockets close (the
// kernel tears down a large address space before it closes the process's files).
static bool proc_dying(int pid) {
  std::string stat;
  if (!read_file("/proc/" + std::to_string(pid) + "/stat", stat)) return true;
  const auto rp = stat.rfind(')');
  if (rp == std::string::npos || rp + 2 >= stat.size()) return true;
  const char state = stat[rp + 2];
  if (state == 'Z' || state == 'X' || state == 'x') return true;
  // fields after the state: ppid pgrp session tty_nr tpgid flags
  unsigned long flags = 0;
  int field = 0;
  size_t i = rp + 3;
  while (i < stat.size() && field < 6) {
    while (i < stat.size() && stat[i] == ' ') i++;
    size_t j = i;
    while (j < stat.size() && stat[j] != ' ') j++;
    if (field == 5) flags = std::strtoul(stat.substr(i, j - i).c_str(), nullptr, 10);
    field++;
    i = j;
  }
  if (flags & 0x4) return true;  // PF_EXITING
  std::string status;
  if (!read_file("/proc/" + std::to_string(pid) + "/status", status)) return true;
  for (const char* key : {"ShdPnd:", "SigPnd:"}) {
    const auto k = status.find(key);
    if (k != std::string::npos && (std::strtoull(status.c_str() + k + 7, nullptr, 16) & (1ull << 8))) return true;
  }
  return false;
}

// The node's GPUs from `nvidia-smi --query-gpu=index,uuid,name,memory.total --format=csv,noheader,nounits`
// (memory in MiB), run as `source` ("nvidia-smi", or another program that answers the same
// query; "none" lists nothing). A node without the program, or whose listing fails, reports none.
std::vector<coord::Device> list_devices(const std::string& source, const std::string& domain) {
  std::vector<coord::Device> out;
  if (source.empty() || source == "none") return out;
  std::string text;
  if (!run_capture({source, "--query-gpu=index,uuid,name,memory.total", "--format=csv,noheader,nounits"}, 20000,
                   text)) {
    ES_WARN("device listing by %s failed: this node reports no devices", source.c_str());
    return out;
  }
  size_t start = 0;
  while (start < text.size()) {
    size_t end = text.find('\n', start);
    if (end == std::string::npos) end = text.size();
    std::string line = text.substr(start, end - start);
    start = end + 1;
    std::vector<std::string> f;
    size_t a = 0;
    for (;;) {
      const size_t c = line.find(',', a);
      std::string x = line.substr(a, c == std::string::npos ? std::string::npos : c - a);
      while (!x.empty() && (x.front() == ' ' || x.front() == '\t')) x.erase(x.begin());
      while (!x.empty() && (x.back() == ' ' || x.back() == '\r' || x.back() == '\t')) x.pop_back();
      f.push_back(x);
      if (c == std::string::npos) break;
      a = c + 1;
    }
    if (f.size() < 4 || f[0].empty() || !std::isdigit((unsigned char)f[0][0])) continue;
    coord::Device d;
    d.index = (uint32_t)std::stoul(f[0]);
    d.uuid = f[1];
    d.class_ = f[2];
    d.memory_bytes = std::isdigit((unsigned char)f[3].c_str()[0]) ? std::stoull(f[3]) << 20 : 0;
    d.domain = domain;
    out.push_back(d);
  }
  return out;
}

// A spare this daemon launched for the coordinator (LaunchSpare) and keeps running: a spare that
// exits before it takes a rank is started again after a backoff (1 s, doubling to 30 s; reset
// after a minute of running). One that took a rank is a worker and no longer supervised.
struct Supervised {
  coord::LaunchSpare spec;
  pid_t pid = 0;
  uint64_t started_ms = 0;
  uint64_t backoff_ms = 1000;
  uint64_t next_start_ms = 0;
  uint32_t starts = 0;
  bool taken = false;
};

struct PendingDelivery {
  coord::Deliver deliver;
  std::set<uint64_t> waiting;  // process connections that owe an Ack
  std::vector<signals::Ack> acks;
  uint64_t deadline_ms = 0;
};

struct Daemon {
  std::string node;
  std::string coordinator;
  uint32_t heartbeat_ms = 500;
  uint64_t ack_timeout_ms = 120000;
  std::string mirror_socket;
  Loop loop;
  std::map<uint64_t, Proc> procs;
  uint64_t coord_conn = 0;
  bool connecting = false;        // a link attempt is in flight on its helper thread
  uint64_t unlinked_at_ms = 0;    // when the last link ended (for the relink time)
  uint64_t term = 0;
  std::deque<std::string> held;  // reports made while unlinked
  std::map<uint64_t, PendingDelivery> deliveries;
  std::map<std::string, uint64_t> epochs;
  uint64_t instance = 0;
  uint64_t backoff_ms = 100;
  std::mt19937_64 rng{std::random_device{}()};
  std::string socket;  // this daemon's process socket (handed to the spares it launches)
  std::string replica_address;  // where this node's store takes replicated rows (announced in the hello)
  std::map<std::string, std::vector<std::string>> replicate_sent;  // engine:rank -> targets told to the store
  std::map<std::string, Supervised> supervised;  // engine:device (or pool/<pool>:device) -> launched spare
  std::vector<coord::Device> devices;            // this node's GPUs, announced in every hello
  std::map<std::string, signals::EnginePlacement> placements;  // the coordinator's latest, by engine
  std::map<std::string, std::set<uint32_t>> departing;  // per engine: the last change's planned departures
  // compile-cache asks waiting for their rank's pair to be placed (answered or refused by deadline)
  struct CacheWait {
    uint64_t conn = 0;
    signals::CacheWanted want;
    uint64_t deadline_ms = 0;
  };
  std::vector<CacheWait> cache_waits;
  uint64_t cache_wait_ms = 600000;

  // ---- up: to the coordinator ------------------------------------------------------------------
  void up(const coord::DaemonToCoord& m) {
    const std::string b = m.serialize();
    if (coord_conn == 0 || !loop.send(coord_conn, b)) {
      held.push_back(b);
      if (held.size() > 10000) held.pop_front();
    }
  }

  coord::EngineState engine_state(const std::string& e) {
    coord::EngineState s;
    s.engine = e;
    s.epoch = epochs[e];
    for (auto& [id, p] : procs) {
      if (!p.registered || p.engine != e) continue;
      if (p.role == signals::Role_ROLE_WORKER) s.workers.push_back(p.rank);
      else if (p.role == signals::Role_ROLE_SPARE) (p.any_rank ? s.any_spares : s.spares).push_back(p.rank);
    }
    return s;
  }

  void send_hello() {
    coord::DaemonToCoord m;
    m.has_hello = true;
    m.hello.node = node;
    m.hello.heartbeat_ms = heartbeat_ms;
    m.hello.protocol = signals::Protocol_PROTOCOL_VERSION;
    m.hello.protocol_oldest = signals::ProtocolOldest_PROTOCOL_OLDEST;
    m.hello.term = term;
    m.hello.mirror_replica_address = replica_address;
    m.hello.devices = devices;
    std::set<std::string> engines;
    for (auto& [id, p] : procs)
      if (p.registered) engines.insert(p.engine);
    for (auto& e : engines) m.hello.engines.push_back(engine_state(e));
    loop.send(coord_conn, m.serialize());
  }

  // The coordinator link: connected on a helper thread (a TCP connect to a dead host would hold
  // the loop for its timeout) and adopted on the loop, with jittered backoff between attempts.
  void link() {
    if (coordinator.empty() || coord_conn != 0 || connecting) return;
    connecting = true;
    const std::string addr = coordinator;
    std::thread([this, addr] {
      Address a;
      std::string err;
      const int fd = Address::parse(addr, a) ? connect_to(a, 1000, &err) : -1;
      loop.post([this, fd] { linked(fd); });
    }).detach();
  }

  void linked(int fd) {
    connecting = false;
    if (fd < 0) {
      metrics().inc("everserve_coordinator_unreachable_total");
      std::uniform_int_distribution<uint64_t> jit(0, backoff_ms / 2);
      const uint64_t wait = backoff_ms + jit(rng);
      backoff_ms = std::min<uint64_t>(backoff_ms * 2, 2000);
      loop.every(wait, [this] { link(); }, false);
      return;
    }
    backoff_ms = 100;
    Conn* c = loop.adopt(fd, coordinator);
    coord_conn = c->id;
    c->on_frame = [this](Conn&, const std::string& f) { from_coordinator(f); };
    c->on_close = [this](Conn&) {
      ES_WARN("coordinator link lost");
      metrics().set("everserve_node_linked", {}, 0);
      metrics().set("everserve_coordinator_linked", {}, 0);
      coord_conn = 0;
      unlinked_at_ms = now_ms();
      loop.every(100, [this] { link(); }, false);
    };
    send_hello();
    while (!held.empty()) {
      loop.send(coord_conn, held.front());
      held.pop_front();
    }
    // a coordinator that took the lease over knows nothing of this node's processes: announce them
    for (auto& [id, p] : procs)
      if (p.registered && registered_kind(p.role) != coord::WorkerEvent_Kind_KIND_UNSPECIFIED)
        worker_event(p, registered_kind(p.role), 0, "");
    metrics().set("everserve_node_linked", {}, 1);
    metrics().set("everserve_coordinator_linked", {}, 1);
    if (unlinked_at_ms) {
      metrics().observe("everserve_coordinator_relink_seconds", {}, (now_ms() - unlinked_at_ms) * 1e-3);
      unlinked_at_ms = 0;
    }
    ES_INFO("linked to coordinator %s", coordinator.c_str());
  }

  // ---- down: from the coordinator --------------------------------------------------------------
  void to_engine(const std::string& engine, const signals::Signal& s, bool workers = true, bool spares = true,
                 bool heads = true) {
    const std::string b = s.serialize();
    for (auto& [id, p] : procs) {
      if (!p.registered || p.engine != engine) continue;
      const bool w = p.role == signals::Role_ROLE_WORKER, sp = p.role == signals::Role_ROLE_SPARE,
                 h = p.role == signals::Role_ROLE_HEAD || p.role == signals::Role_ROLE_CLIENT;
      if ((w && workers) || (sp && spares) || (h && heads)) loop.send(id, b);
    }
  }

  void from_coordinator(const std::string& frame) {
    coord::CoordToDaemon m;
    if (!m.parse(frame)) {
      ES_WARN("malformed coordinator message");
      return;
    }
    if (m.term < term) return;  // an old coordinator: fenced
    term = std::max(term, m.term);
    if (m.has_deliver) {
      departing[m.deliver.engine] = std::set<uint32_t>(m.deliver.change.departing.begin(), m.deliver.change.departing.end());
      deliver(m.deliver);
    } else if (m.has_committed) {
      epochs[m.committed.engine] = std::max(epochs[m.committed.engine], m.committed.membership.epoch);
      signals::Signal s;
      s.has_membership_committed = true;
      s.membership_committed = m.committed.membership;
      to_engine(m.committed.engine, s);
      // a spare that took a rank is a worker of the new membership
      for (auto& t : m.committed.take)
        for (auto& [id, p] : procs)
          if (p.registered && p.engine == m.committed.engine && p.role == signals::Role_ROLE_SPARE &&
              (p.rank == t.rank || p.any_rank) && t.node == node && (t.device == p.device)) {
            p.role = signals::Role_ROLE_WORKER;
            for (auto& [key, sv] : supervised)
              if (sv.pid != 0 && (uint32_t)sv.pid == p.pid) sv.taken = true;
            p.rank = t.rank;
            p.any_rank = false;
            break;
          }
      fence_displaced(m.committed);
    } else if (m.has_abandon) {
      signals::Signal s;
      s.has_abandoned = true;
      s.abandoned.epoch = m.abandon.epoch;
      s.abandoned.detail = m.abandon.detail;
      to_engine(m.abandon.engine, s);
    } else if (m.has_forward_change) {
      signals::Signal s;
      s.has_change = true;
      s.change = m.forward_change.change;
      to_engine(m.forward_change.engine, s, false, false, true);
    } else if (m.has_forward_notice) {
      signals::Signal s;
      s.has_notice = true;
      s.notice = m.forward_notice.notice;
      to_engine(m.forward_notice.engine, s);
    } else if (m.has_forward_join) {
      signals::Signal s;
      s.has_join = true;
      s.join = m.forward_join.join;
      if (m.forward_join.to_clients) {
        to_engine(m.forward_join.engine, s, false, false, true);
      } else {
        for (auto& [id, p] : procs)
          if (p.registered && p.engine == m.forward_join.engine && p.rank == m.forward_join.join.rank &&
              (p.role == signals::Role_ROLE_WORKER || p.role == signals::Role_ROLE_SPARE))
            loop.send(id, s.serialize());
      }
    } else if (m.has_cover_plan) {
      signals::Signal s;
      s.has_cover_plan = true;
      s.cover_plan = m.cover_plan;
      to_engine(m.cover_plan.engine, s);
    } else if (m.has_group_id) {
      signals::Signal s;
      s.has_group_id = true;
      s.group_id = m.group_id;
      to_engine(m.group_id.engine, s);
    } else if (m.has_engine_policy) {
      signals::Signal s;
      s.has_engine_policy = true;
      s.engine_policy = m.engine_policy;
      to_engine(m.engine_policy.engine, s);
    } else if (m.has_engine_placement) {
      placements[m.engine_placement.engine] = m.engine_placement;
      answer_cache_waits(m.engine_placement.engine);
      signals::Signal s;
      s.has_engine_placement = true;
      s.engine_placement = m.engine_placement;
      to_engine(m.engine_placement.engine, s);
    } else if (m.has_instance_state) {
      signals::Signal s;
      s.has_instance_state = true;
      s.instance_state = m.instance_state;
      to_engine(m.instance_state.engine, s, false, false, true);
    } else if (m.has_role_answer) {
      for (auto& [id, p] : procs)
        if (p.engine == m.role_answer.engine && p.role == signals::Role_ROLE_UNDECIDED) {
          signals::Signal s;
          s.has_role_assigned = true;
          s.role_assigned.engine = m.role_answer.engine;
          s.role_assigned.rank = m.role_answer.rank;
          s.role_assigned.epoch = m.role_answer.epoch;
          s.role_assigned.role = m.role_answer.role;
          s.role_assigned.refusal = m.role_answer.refusal;
          loop.send(id, s.serialize());
          if (m.role_answer.refusal.empty()) {
            p.role = m.role_answer.role;
            p.rank = m.role_answer.rank;
          }
          break;
        }
    } else if (m.has_stacks) {
      for (auto& [id, p] : procs)
        if (p.registered && p.engine == m.stacks.engine && (!m.stacks.has_rank || p.rank == m.stacks.rank)) {
          signals::Signal s;
          s.has_dump_stacks = true;
          s.dump_stacks.request_id = m.stacks.request_id;
          s.dump_stacks.reason = "operator";
          loop.send(id, s.serialize());
        }
    } else if (m.has_replay_ask || m.has_replay_offer) {
      signals::Signal s;
      if (m.has_replay_ask) {
        s.has_replay_ask = true;
        s.replay_ask = m.replay_ask;
        to_engine(m.replay_ask.engine, s, false, false, true);
      } else {
        // an offer goes to the connection that asked (its ProcessRef), registered or not
        s.has_replay_offer = true;
        s.replay_offer = m.replay_offer;
        const auto& to = m.replay_offer.to;
        if (to.node == node && to.instance == instance && procs.count(to.serial)) loop.send(to.serial, s.serialize());
      }
    } else if (m.has_launch_spare) {
      launch_spare(m.launch_spare);
    } else if (m.has_replicate_targets) {
      replicate(m.replicate_targets);
    }
  }

  void deliver(const coord::Deliver& d) {
    PendingDelivery pd;
    pd.deliver = d;
    pd.deadline_ms = now_ms() + ack_timeout_ms;
    signals::Signal s;
    s.has_change = true;
    s.change = d.change;
    s.change.delivered_at_us = now_us();
    const std::string b = s.serialize();
    for (auto& [id, p] : procs) {
      if (!p.registered || p.engine != d.engine) continue;
      bool named = false;
      if (p.role == signals::Role_ROLE_WORKER)
        named = std::find(d.to_ranks.begin(), d.to_ranks.end(), p.rank) != d.to_ranks.end();
      else if (p.role == signals::Role_ROLE_SPARE)
        named = std::any_of(d.take.begin(), d.take.end(), [&](const signals::Take& t) {
          return (t.rank == p.rank || p.any_rank) && t.node == node && t.device == p.device;
        });
      if (named) {
        loop.send(id, b);
        pd.waiting.insert(id);
      } else if (p.role == signals::Role_ROLE_HEAD || p.role == signals::Role_ROLE_CLIENT) {
        loop.send(id, b);  // the head learns of the change to cut its step; it does not ack
      }
    }
    deliveries[d.request_id] = std::move(pd);
    maybe_delivered(d.request_id);
  }

  void maybe_delivered(uint64_t rid, const std::string& error = "") {
    auto it = deliveries.find(rid);
    if (it == deliveries.end()) return;
    if (!it->second.waiting.empty() && error.empty()) return;
    coord::DaemonToCoord m;
    m.has_delivered = true;
    m.delivered.request_id = rid;
    m.delivered.engine = it->second.deliver.engine;
    m.delivered.epoch = it->second.deliver.change.epoch;
    m.delivered.acks = it->second.acks;
    m.delivered.error = error;
    deliveries.erase(it);
    up(m);
  }

  // ---- processes -------------------------------------------------------------------------------
  void worker_event(const Proc& p, int32_t kind, int32_t cause, const std::string& detail) {
    coord::DaemonToCoord m;
    m.has_worker_event = true;
    auto& ev = m.worker_event;
    ev.engine = p.engine;
    ev.kind = kind;
    ev.rank = p.rank;
    ev.device = p.device;
    ev.pid = p.pid;
    ev.launcher_pid = p.reg.launcher_pid;
    ev.any_rank = p.any_rank;
    ev.cause = cause;
    ev.detail = detail;
    ev.epoch = epochs[p.engine];
    ev.host = p.reg.host;
    if (p.reg.has_identity) {
      ev.identity = p.reg.identity;
      ev.has_identity = true;
    }
    if (p.reg.has_compile_cache) {
      ev.compile_cache = p.reg.compile_cache;
      ev.has_compile_cache = true;
    }
    ev.has_connection = true;
    ev.connection.instance = instance;
    ev.connection.serial = p.conn;
    ev.connection.pid = p.pid;
    up(m);
  }

  static int32_t registered_kind(int32_t role) {
    switch (role) {
      case signals::Role_ROLE_WORKER: return coord::WorkerEvent_Kind_WORKER_REGISTERED;
      case signals::Role_ROLE_SPARE: return coord::WorkerEvent_Kind_SPARE_REGISTERED;
      case signals::Role_ROLE_HEAD: return coord::WorkerEvent_Kind_HEAD_REGISTERED;
      default: return coord::WorkerEvent_Kind_KIND_UNSPECIFIED;
    }
  }
  static int32_t departed_kind(int32_t role) {
    switch (role) {
      case signals::Role_ROLE_WORKER: return coord::WorkerEvent_Kind_WORKER_DEPARTED;
      case signals::Role_ROLE_SPARE: return coord::WorkerEvent_Kind_SPARE_DEPARTED;
      case signals::Role_ROLE_HEAD: return coord::WorkerEvent_Kind_HEAD_DEPARTED;
      case signals::Role_ROLE_UNDECIDED: return coord::WorkerEvent_Kind_UNDECIDED_DEPARTED;
      default: return coord::WorkerEvent_Kind_KIND_UNSPECIFIED;
    }
  }

  void from_process(Conn& c, const std::string& frame) {
    signals::Signal s;
    if (!s.parse(frame)) {
      ES_WARN("malformed signal from a process");
      return;
    }
    Proc& p = procs[c.id];
    p.conn = c.id;
    if (s.has_register) {
      const auto& r = s.register_;
      if (r.protocol != 0 && r.protocol < signals::ProtocolOldest_PROTOCOL_OLDEST) {
        signals::Signal g;
        g.has_goodbye = true;
        g.goodbye.cause = signals::StopCause_STOP_CAUSE_REFUSED;
        g.goodbye.detail = "protocol " + std::to_string(r.protocol) + " is older than this daemon's oldest";
        loop.send(c.id, g.serialize());
        return;
      }
      p.engine = r.engine;
      p.rank = r.rank;
      p.role = r.role;
      p.any_rank = r.any_rank;
      p.pid = r.launcher_pid;
      p.device = r.has_member ? r.member.device : 0;
      p.reg = r;
      p.registered = true;
      {
        ucred cred{};
        socklen_t len = sizeof(cred);
        if (getsockopt(c.fd, SOL_SOCKET, SO_PEERCRED, &cred, &len) == 0 && cred.pid > 0) p.os_pid = cred.pid;
      }
      metrics().inc("everserve_node_registrations_total", {{"role", std::to_string(r.role)}});
      if (r.role == signals::Role_ROLE_UNDECIDED) {
        coord::DaemonToCoord m;
        m.has_role_asked = true;
        m.role_asked.request_id = c.id;
        m.role_asked.engine = r.engine;
        m.role_asked.rank = r.rank;
        m.role_asked.host = r.host;
        up(m);
      } else if (r.role != signals::Role_ROLE_CLIENT) {
        worker_event(p, registered_kind(r.role), 0, "");
      }
      ES_INFO("registered %s rank %u role %d (conn %llu)", r.engine.c_str(), r.rank, r.role,
              (unsigned long long)c.id);
    } else if (s.has_ack) {
      for (auto& [rid, pd] : deliveries) {
        if (pd.waiting.erase(c.id)) {
          signals::Ack a = s.ack;
          a.received_at_us = now_us();
          pd.acks.push_back(a);
          if (!a.error.empty()) {
            maybe_delivered(rid, "rank " + std::to_string(a.rank) + ": " + a.error);
          } else {
            maybe_delivered(rid);
          }
          break;
        }
      }
    } else if (s.has_rank_lost) {
      coord::DaemonToCoord m;
      m.has_lost_report = true;
      m.lost_report.engine = p.engine;
      m.lost_report.lost = s.rank_lost;
      m.lost_report.has_lost = true;
      up(m);
    } else if (s.has_notice) {
      coord::DaemonToCoord m;
      m.has_notice_report = true;
      m.notice_report.engine = p.engine;
      m.notice_report.notice = s.notice;
      m.notice_report.has_notice = true;
      up(m);
    } else if (s.has_join) {
      coord::DaemonToCoord m;
      m.has_join_report = true;
      m.join_report.engine = s.join.engine.empty() ? p.engine : s.join.engine;
      m.join_report.join = s.join;
      m.join_report.has_join = true;
      m.join_report.from_client = p.role == signals::Role_ROLE_HEAD || p.role == signals::Role_ROLE_CLIENT;
      up(m);
    } else if (s.has_goodbye) {
      p.said_goodbye = true;
      p.goodbye_cause = s.goodbye.cause ? s.goodbye.cause : signals::StopCause_STOP_CAUSE_STOPPED;
    } else if (s.has_group_formed || s.has_group_failed || s.has_group_released || s.has_group_ready) {
      coord::DaemonToCoord m;
      m.has_cover_report = true;
      if (s.has_group_formed) {
        m.cover_report.has_formed = true;
        m.cover_report.formed = s.group_formed;
      } else if (s.has_group_failed) {
        m.cover_report.has_failed = true;
        m.cover_report.failed = s.group_failed;
      } else if (s.has_group_released) {
        m.cover_report.has_released = true;
        m.cover_report.released = s.group_released;
      } else {
        m.cover_report.has_ready = true;
        m.cover_report.ready = s.group_ready;
      }
      up(m);
    } else if (s.has_group_id) {
      coord::DaemonToCoord m;
      m.has_group_id = true;
      m.group_id = s.group_id;
      up(m);
    } else if (s.has_release_leaked) {
      coord::DaemonToCoord m;
      m.has_release_leaked = true;
      m.release_leaked.leak = s.release_leaked;
      m.release_leaked.has_leak = true;
      up(m);
    } else if (s.has_stacks_dumped) {
      coord::DaemonToCoord m;
      m.has_stacks_sent = true;
      m.stacks_sent.request_id = s.stacks_dumped.request_id;
      m.stacks_sent.pid = p.pid;
      m.stacks_sent.answered = true;
      m.stacks_sent.text = s.stacks_dumped.text.substr(0, 1 << 20);
      up(m);
    } else if (s.has_cache_wanted) {
      CacheWait w;
      w.conn = c.id;
      w.want = s.cache_wanted;
      w.deadline_ms = now_ms() + cache_wait_ms;
      cache_waits.push_back(w);
      answer_cache_waits(w.want.engine);
    } else if (s.has_replay_ask || s.has_replay_offer) {
      coord::DaemonToCoord m;
      if (s.has_replay_ask) {
        m.has_replay_ask = true;
        m.replay_ask = s.replay_ask;
        m.replay_ask.asker.node = node;  // where the offer must come back to
        m.replay_ask.asker.instance = instance;
        m.replay_ask.asker.serial = c.id;
        m.replay_ask.has_asker = true;
      } else {
        m.has_replay_offer = true;
        m.replay_offer = s.replay_offer;
      }
      up(m);
    }
  }

  void process_closed(Conn& c) {
    auto it = procs.find(c.id);
    if (it == procs.end()) return;
    Proc p = it->second;
    procs.erase(it);
    // a named process that went away owes no Ack any more: report the delivery with an error
    for (auto& [rid, pd] : deliveries)
      if (pd.waiting.erase(c.id)) {
        signals::Ack a;
        a.rank = p.rank;
        a.epoch = pd.deliver.change.epoch;
        a.error = "process departed before its ack";
        pd.acks.push_back(a);
        maybe_delivered(rid, "rank " + std::to_string(p.rank) + " departed during the change");
        break;
      }
    if (p.registered && p.role != signals::Role_ROLE_CLIENT && !p.reported_gone)
      worker_event(p, departed_kind(p.role), p.said_goodbye ? p.goodbye_cause : signals::StopCause_STOP_CAUSE_LOST,
                   p.said_goodbye ? "goodbye" : "connection ended");
  }

  // ---- the process watcher: a dying worker is reported before its connection closes --------------
  void watch_processes() {
    for (auto& [id, p] : procs) {
      if (!p.registered || p.reported_gone || p.os_pid <= 0 || p.said_goodbye) continue;
      if (p.role != signals::Role_ROLE_WORKER && p.role != signals::Role_ROLE_SPARE) continue;
      if (!proc_dying(p.os_pid)) continue;
      p.reported_gone = true;
      metrics().inc("everserve_node_processes_lost_total", {{"engine", p.engine}});
      ES_WARN("process %d (%s rank %u) is exiting: reported lost", p.os_pid, p.engine.c_str(), p.rank);
      worker_event(p, departed_kind(p.role), signals::StopCause_STOP_CAUSE_LOST, "process exiting");
      for (auto& [rid, pd] : deliveries)
        if (pd.waiting.erase(id)) {
          signals::Ack a;
          a.rank = p.rank;
          a.epoch = pd.deliver.change.epoch;
          a.error = "process departed before its ack";
          pd.acks.push_back(a);
          maybe_delivered(rid, "rank " + std::to_string(p.rank) + " departed during the change");
          break;
        }
    }
  }

  // ---- replication targets: the coordinator names which stores take a rank's rows --------------
  void replicate(const coord::ReplicateTargets& t) {
    if (mirror_socket.empty()) return;
    const std::string key = t.engine + ":" + std::to_string(t.rank);
    if (replicate_sent[key] == t.targets) return;
    mirror::MirrorRequest req;
    req.has_replicate = true;
    req.replicate.engine = t.engine;
    req.replicate.rank = t.rank;
    req.replicate.targets = t.targets;
    req.replicate.node = node;
    Address a;
    std::string err, reply;
    int fd = -1;
    if (Address::parse(mirror_socket, a)) fd = connect_to(a, 1000, &err);
    if (fd < 0) {
      ES_WARN("replication targets for %s: store unreachable (%s)", key.c_str(), err.c_str());
      return;
    }
    if (write_frame(fd, req.serialize()) && read_frame(fd, reply, 2000)) replicate_sent[key] = t.targets;
    ::close(fd);
    ES_INFO("store of %s replicates %s to %zu target(s)", node.c_str(), key.c_str(), t.targets.size());
  }

  // ---- fencing: a worker of this node whose rank the commit gave away, still running -------------
  // A lost rank that did not leave by notice and whose process is still connected is hung or cut
  // off; its position now belongs to another process. It is stopped (SIGTERM, SIGKILL after
  // 5 s) so it can write nothing more and its GPU is free again. Planned departures finish their
  // step and are released by the head; they are left alone.
  void fence_displaced(const coord::Committed& c) {
    const auto& gone = departing[c.engine];
    for (uint32_t r : c.lost) {
      if (gone.count(r)) continue;
      const signals::Take* take = nullptr;
      for (auto& t : c.take)
        if (t.rank == r) take = &t;
      for (auto& [id, p] : procs) {
        if (!p.registered || p.engine != c.engine || p.rank != r || p.role != signals::Role_ROLE_WORKER ||
            p.os_pid <= 0)
          continue;
        if (take != nullptr && take->node == node && take->device == p.device) continue;  // the new holder
        const pid_t pid = (pid_t)p.os_pid;
        ES_WARN("fencing %s rank %u (process %d): the commit to epoch %llu gave its position away", c.engine.c_str(),
                r, (int)pid, (unsigned long long)c.membership.epoch);
        metrics().inc("everserve_node_fenced_total", {{"engine", c.engine}});
        kill(pid, SIGTERM);
        loop.every(5000, [pid] {
          if (kill(pid, 0) == 0) kill(pid, SIGKILL);
        }, false);
      }
    }
  }

  // ---- compile caches: a spare's rank's artifacts, fetched into this node's store ----------------
  void cache_answer(uint64_t conn, const signals::CacheWanted& want, bool ok, const signals::CompileCache& pair,
                    const std::string& why) {
    signals::Signal s;
    if (ok) {
      s.has_cache_ready = true;
      s.cache_ready.engine = want.engine;
      s.cache_ready.rank = want.rank;
      s.cache_ready.key = pair.key;
      s.cache_ready.digest = pair.digest;
    } else {
      s.has_cache_refused = true;
      s.cache_refused.engine = want.engine;
      s.cache_refused.rank = want.rank;
      s.cache_refused.reason = why;
      ES_WARN("%s: rank %u's compile cache: %s", want.engine.c_str(), want.rank, why.c_str());
    }
    metrics().inc("everserve_node_cache_asks_total", {{"verdict", ok ? "ready" : "refused"}});
    loop.send(conn, s.serialize());
  }

  // Answer the asks of `engine` whose rank's pair is placed (its set fetched by the node's store
  // from the stores holding it, on a thread of its own), and refuse those past their deadline.
  void answer_cache_waits(const std::string& engine) {
    const uint64_t now = now_ms();
    std::vector<CacheWait> keep;
    for (auto& w : cache_waits) {
      if (!procs.count(w.conn)) continue;  // the asker left
      const signals::RankPlacement* rp = nullptr;
      auto pit = placements.find(w.want.engine);
      if (pit != placements.end())
        for (auto& m : pit->second.members)
          if (m.rank == w.want.rank && m.has_compile_cache && !m.compile_cache.key.empty()) rp = &m;
      if (rp == nullptr) {
        if (now >= w.deadline_ms) cache_answer(w.conn, w.want, false, {}, "no compile-cache pair placed for the rank in time");
        else keep.push_back(w);
        continue;
      }
      if (w.want.engine != engine && !engine.empty()) {
        keep.push_back(w);
        continue;
      }
      if (mirror_socket.empty()) {
        cache_answer(w.conn, w.want, false, {}, "this node has no store to fetch it into");
        continue;
      }
      mirror::MirrorRequest req;
      req.has_cache_fetch = true;
      req.cache_fetch.key = rp->compile_cache.key;
      req.cache_fetch.digest = rp->compile_cache.digest;
      req.cache_fetch.rank = w.want.rank;
      req.cache_fetch.dp = w.want.dp;
      req.cache_fetch.holders = rp->cache_holders;
      const signals::CompileCache pair = rp->compile_cache;
      const std::string store = mirror_socket;
      const uint64_t conn = w.conn;
      const signals::CacheWanted want = w.want;
      const int timeout_ms = (int)std::max<int64_t>(1000, (int64_t)w.deadline_ms - (int64_t)now);
      std::thread([this, req, pair, store, conn, want, timeout_ms] {
        Address a;
        std::string err, reply;
        bool ok = false;
        const int fd = Address::parse(store, a) ? connect_to(a, 2000, &err) : -1;
        if (fd >= 0) {
          mirror::MirrorReply r;
          if (write_frame(fd, req.serialize()) && read_frame(fd, reply, timeout_ms) && r.parse(reply)) {
            ok = r.error.empty();
            err = r.error;
          } else if (err.empty()) {
            err = "the store did not answer";
          }
          ::close(fd);
        }
        loop.post([this, conn, want, ok, pair, err] {
          if (procs.count(conn)) cache_answer(conn, want, ok, pair, err);
        });
      }).detach();
    }
    cache_waits = std::move(keep);
  }

  // ---- spares launched for the coordinator -----------------------------------------------------
  void launch_spare(const coord::LaunchSpare& spec) {
    const std::string key = (spec.pool.empty() ? spec.engine : "pool/" + spec.pool) + ":" + std::to_string(spec.device);
    if (spec.command.empty()) return;
    auto it = supervised.find(key);
    if (it != supervised.end() && !it->second.taken) return;  // already standing (or starting)
    Supervised sv;
    sv.spec = spec;
    supervised[key] = sv;
    start_spare(supervised[key]);
  }

  // `{pool}`, `{device}`, `{node}`, `{socket}`, `{engines}`, `{engine}` and `{rank}` in a launch's
  // command and environment.
  std::string fill(std::string s, const coord::LaunchSpare& spec) const {
    std::string engines_csv;
    for (size_t i = 0; i < spec.engines.size(); i++) engines_csv += (i ? "," : "") + spec.engines[i];
    if (engines_csv.empty()) engines_csv = spec.engine;
    const std::pair<const char*, std::string> subs[] = {
        {"{pool}", spec.pool}, {"{device}", std::to_string(spec.device)}, {"{node}", node}, {"{socket}", socket},
        {"{engines}", engines_csv}, {"{engine}", spec.engine}, {"{rank}", spec.has_rank ? std::to_string(spec.rank) : ""}};
    for (auto& [k, v] : subs)
      for (size_t at = s.find(k); at != std::string::npos; at = s.find(k, at + v.size())) s.replace(at, strlen(k), v);
    return s;
  }

  void start_spare(Supervised& sv) {
    std::vector<std::string> envs;
    for (char** e = environ; *e; e++) envs.emplace_back(*e);
    auto set = [&](const std::string& k, const std::string& v) { envs.push_back(k + "=" + v); };
    for (auto& [k, v] : sv.spec.env) set(k, fill(v, sv.spec));
    std::string engines_csv;
    for (size_t i = 0; i < sv.spec.engines.size(); i++) engines_csv += (i ? "," : "") + sv.spec.engines[i];
    set("EVERSERVE_ENGINES", engines_csv.empty() ? sv.spec.engine : engines_csv);
    if (!sv.spec.pool.empty()) set("EVERSERVE_POOL", sv.spec.pool);
    set("EVERSERVE_ENGINE", sv.spec.engine);
    set("EVERSERVE_SPARE_RANK", sv.spec.has_rank ? std::to_string(sv.spec.rank) : "any");
    set("EVERSERVE_DEVICE", std::to_string(sv.spec.device));
    set("EVERSERVE_SOCKET", socket);
    set("EVERSERVE_NODE", node);
    if (!mirror_socket.empty()) set("EVERSERVE_MIRROR_SOCKET", mirror_socket);
    const pid_t pid = fork();
    if (pid < 0) {
      ES_ERROR("cannot fork a spare for %s", sv.spec.engine.c_str());
      sv.next_start_ms = now_ms() + sv.backoff_ms;
      return;
    }
    if (pid == 0) {
      setpgid(0, 0);
      std::vector<std::string> args;
      for (auto& a : sv.spec.command) args.push_back(fill(a, sv.spec));
      std::vector<char*> argv, envp;
      for (auto& a : args) argv.push_back(const_cast<char*>(a.c_str()));
      argv.push_back(nullptr);
      for (auto& e : envs) envp.push_back(const_cast<char*>(e.c_str()));
      envp.push_back(nullptr);
      execvpe(argv[0], argv.data(), envp.data());
      _exit(127);
    }
    sv.pid = pid;
    sv.started_ms = now_ms();
    sv.starts++;
    metrics().inc("everserve_node_spare_starts_total", {{"engine", sv.spec.engine}});
    ES_INFO("launched a spare for %s on device %u (pid %d, start %u)", sv.spec.engine.c_str(), sv.spec.device, (int)pid,
            sv.starts);
  }

  void supervise() {
    int status = 0;
    pid_t pid;
    while ((pid = waitpid(-1, &status, WNOHANG)) > 0) {
      for (auto& [key, sv] : supervised) {
        if (sv.pid != pid) continue;
        sv.pid = 0;
        if (sv.taken) break;
        const uint64_t ran = now_ms() - sv.started_ms;
        if (ran > 60000) sv.backoff_ms = 1000;
        sv.next_start_ms = now_ms() + sv.backoff_ms;
        ES_WARN("spare of %s on device %u exited (status %d) after %llu ms; again in %llu ms", sv.spec.engine.c_str(),
                sv.spec.device, status, (unsigned long long)ran, (unsigned long long)sv.backoff_ms);
        sv.backoff_ms = std::min<uint64_t>(sv.backoff_ms * 2, 30000);
        break;
      }
    }
    const uint64_t now = now_ms();
    for (auto& [key, sv] : supervised)
      if (!sv.taken && sv.pid == 0 && now >= sv.next_start_ms) start_spare(sv);
  }

  void stop_spares() {
    for (auto& [key, sv] : supervised)
      if (sv.pid > 0 && !sv.taken) kill(-sv.pid, SIGTERM);
  }

  void tick() {
    if (!cache_waits.empty()) answer_cache_waits("");
    if (coord_conn != 0) {
      coord::DaemonToCoord m;
      m.has_heartbeat = true;
      loop.send(coord_conn, m.serialize());
    }
    const uint64_t now = now_ms();
    std::vector<uint64_t> expired;
    for (auto& [rid, pd] : deliveries)
      if (now > pd.deadline_ms) expired.push_back(rid);
    for (auto rid : expired) maybe_delivered(rid, "acks timed out");
    uint64_t workers = 0;
    for (auto& [id, p] : procs) workers += p.registered && p.role == signals::Role_ROLE_WORKER;
    metrics().set("everserve_node_workers", {}, (double)workers);
  }
};

}  // namespace

int main(int argc, char** argv) {
  std::string enroll_url = env_or("EVERSERVE_ENROLL_URL", "");
  std::string tls_dir = env_or("EVERSERVE_TLS_DIR", "");
  for (int i = 1; i + 1 < argc; i += 2) {
    if (std::string(argv[i]) == "--enroll") enroll_url = argv[i + 1];
    if (std::string(argv[i]) == "--tls-dir") tls_dir = argv[i + 1];
  }
  if (enroll_url.empty()) {
    std::string terr;
    if (!es::tls::configure_from_env(&terr)) {
      fprintf(stderr, "TLS: %s\n", terr.c_str());
      return 2;
    }
  }
  log_init("node");
  signal(SIGPIPE, SIG_IGN);
  Daemon d;
  d.node = env_or("EVERSERVE_NODE", "node0");
  std::string socket = env_or("EVERSERVE_SOCKET", "unix:/tmp/everserve-node.sock");
  d.coordinator = env_or("EVERSERVE_COORDINATOR", "");
  d.heartbeat_ms = (uint32_t)std::stoul(env_or("EVERSERVE_HEARTBEAT_MS", "500"));
  d.mirror_socket = env_or("EVERSERVE_MIRROR_SOCKET", "");
  std::string metrics_addr = env_or("EVERSERVE_METRICS_ADDR", "");
  std::string discovery = env_or("EVERSERVE_DISCOVERY_DIR", "");
  std::string notice_source = env_or("EVERSERVE_NOTICE_SOURCE", "");
  std::string notice_endpoint = env_or("EVERSERVE_NOTICE_ENDPOINT", "");
  uint32_t notice_interval = 1000;
  uint64_t proc_poll_ms = std::stoull(env_or("EVERSERVE_PROC_POLL_MS", "2"));
  std::string devices_from = env_or("EVERSERVE_DEVICES_FROM", "nvidia-smi");
  std::string domain = env_or("EVERSERVE_DOMAIN", "");
  for (int i = 1; i + 1 < argc; i += 2) {
    const std::string k = argv[i], v = argv[i + 1];
    if (k == "--node") d.node = v;
    else if (k == "--socket") socket = v;
    else if (k == "--coordinator") d.coordinator = v;
    else if (k == "--heartbeat-ms") d.heartbeat_ms = (uint32_t)std::stoul(v);
    else if (k == "--ack-timeout-ms") d.ack_timeout_ms = std::stoull(v);
    else if (k == "--metrics-addr") metrics_addr = v;
    else if (k == "--mirror-socket") d.mirror_socket = v;
    else if (k == "--discovery-dir") discovery = v;
    else if (k == "--replica-address") d.replica_address = v;
    else if (k == "--proc-poll-ms") proc_poll_ms = std::stoull(v);
    else if (k == "--notice-source") notice_source = v;
    else if (k == "--notice-endpoint") notice_endpoint = v;
    else if (k == "--notice-interval-ms") notice_interval = (uint32_t)std::stoul(v);
    else if (k == "--devices-from") devices_from = v;
    else if (k == "--domain") domain = v;
    else if (k == "--cache-wait-ms") d.cache_wait_ms = std::stoull(v);
    else if (k == "--enroll" || k == "--tls-dir") continue;  // read above
    else {
      fprintf(stderr, "unknown flag %s\n", k.c_str());
      return 2;
    }
  }
  if (!enroll_url.empty()) {
    // the node's certificate from the coordinator's issuer, then mutual TLS with it
    if (tls_dir.empty()) {
      ES_ERROR("--enroll needs --tls-dir (holding the bootstrap ca.crt)");
      return 2;
    }
    const std::string token_file = env_or("EVERSERVE_ENROLL_TOKEN_FILE", "/var/run/secrets/everserve/token");
    Enrolled held;
    if (!enrolled_in(tls_dir, 600000, held)) {
      std::string e;
      bool ok = false;
      const int attempts = std::stoi(env_or("EVERSERVE_ENROLL_ATTEMPTS", "5"));
      for (int attempt = 0; attempt < attempts && !(ok = enroll(enroll_url, tls_dir, token_file, held, e)); attempt++) {
        ES_WARN("enrollment: %s", e.c_str());
        if (attempt + 1 < attempts) sleep(1u << std::min(attempt, 5));
      }
      if (!ok) {
        ES_ERROR("enrollment at %s failed: %s", enroll_url.c_str(), e.c_str());
        return 2;
      }
    }
    if (held.node != d.node) ES_WARN("the certificate names node %s, not %s", held.node.c_str(), d.node.c_str());
    std::string terr;
    tls::Config tc{tls_dir + "/ca.crt", tls_dir + "/node.crt", tls_dir + "/node.key"};
    if (!tls::configure(tc, &terr)) {
      ES_ERROR("TLS: %s", terr.c_str());
      return 2;
    }
    ES_INFO("enrolled as %s until %lld", held.node.c_str(), (long long)held.not_after_ms);
    // renew at half the certificate's life; the new files are taken on the loop's thread
    std::thread([enroll_url, tls_dir, token_file, held, &d]() mutable {
      for (;;) {
        const int64_t half = held.issued_at_ms + (held.not_after_ms - held.issued_at_ms) / 2;
        const int64_t wait = std::max<int64_t>(30000, half - wall_clock_ms());
        std::this_thread::sleep_for(std::chrono::milliseconds(wait));
        std::string e;
        if (!enroll(enroll_url, tls_dir, token_file, held, e)) {
          ES_WARN("renewal: %s", e.c_str());
          held.issued_at_ms = wall_clock_ms() - (held.not_after_ms - wall_clock_ms());  // again in 30 s
          continue;
        }
        d.loop.post([tls_dir] {
          std::string terr;
          if (!tls::configure({tls_dir + "/ca.crt", tls_dir + "/node.crt", tls_dir + "/node.key"}, &terr))
            ES_ERROR("TLS after renewal: %s", terr.c_str());
          else
            ES_INFO("certificate renewed");
        });
      }
    }).detach();
  }
  d.instance = (now_us() << 8) ^ (uint64_t)getpid();
  d.socket = socket;
  d.devices = list_devices(devices_from, domain);
  ES_INFO("%zu device(s) on %s", d.devices.size(), d.node.c_str());
  metrics().describe("everserve_node_linked", "1 while the daemon is linked to the coordinator", "gauge");
  metrics().describe("everserve_node_fenced_total", "Displaced workers this daemon stopped after a commit", "counter");
  metrics().describe("everserve_coordinator_linked", "1 while the daemon is linked to the coordinator", "gauge");
  metrics().describe("everserve_coordinator_relink_seconds", "From a lost coordinator link to the next one", "histogram");
  metrics().describe("everserve_coordinator_unreachable_total", "Link attempts the coordinator did not answer", "counter");
  metrics().describe("everserve_node_workers", "Workers registered on this node", "gauge");
  Address a;
  std::string err;
  if (!Address::parse(socket, a) || !d.loop.listen(a, [&](Conn& c) {
        c.on_frame = [&](Conn& cc, const std::string& f) { d.from_process(cc, f); };
        c.on_close = [&](Conn& cc) { d.process_closed(cc); };
      }, &err)) {
    ES_ERROR("listen %s: %s", socket.c_str(), err.c_str());
    return 1;
  }
  if (!discovery.empty()) {
    // the discovery record (discovery.proto DaemonRecord in proto3 JSON) for processes that look
    // their node's daemon up
    mkdirs(discovery);
    const std::string rec = "{\"node\":\"" + json_escape(d.node) + "\",\"address\":\"" + json_escape(socket) +
                            "\",\"startedAtMs\":\"" + std::to_string(now_ms()) + "\",\"pid\":" +
                            std::to_string(getpid()) + ",\"mirrorAddress\":\"" + json_escape(d.mirror_socket) + "\"}";
    write_file_atomic(discovery + "/" + d.node + ".json", rec);
  }
  if (!metrics_addr.empty() && !serve_http(d.loop, metrics_addr, nullptr, &err)) {
    ES_ERROR("metrics %s: %s", metrics_addr.c_str(), err.c_str());
    return 1;
  }
  d.loop.every(tls::reload_period_ms(), [] {  // renewed certificates, taken without a restart
    std::string terr;
    if (!tls::reload_if_changed(&terr)) ES_WARN("TLS reload: %s", terr.c_str());
  });
  d.link();
  d.loop.every(d.heartbeat_ms, [&] { d.tick(); });
  d.loop.every(100, [&] { d.supervise(); });
  d.loop.every(proc_poll_ms, [&] { d.watch_processes(); });
  std::unique_ptr<NoticeWatcher> notices;
  if (!notice_source.empty()) {
    notices = std::make_unique<NoticeWatcher>(notice_source, notice_endpoint, d.node, notice_interval);
    if (!notices->start(&err)) {
      ES_ERROR("%s", err.c_str());
      return 2;
    }
    d.loop.every(100, [&] {
      NodeNoticeEvent ev;
      if (!notices->take(ev)) return;
      ES_WARN("node notice from %s: %s (deadline %lld)", ev.source.c_str(), ev.detail.c_str(), (long long)ev.deadline_ms);
      coord::DaemonToCoord m;
      m.has_node_notice = true;
      m.node_notice.deadline_ms = ev.deadline_ms;
      m.node_notice.reason = signals::Reason_REASON_NOTICE;
      m.node_notice.source = ev.source;
      m.node_notice.detail = ev.detail;
      d.up(m);
    });
  }
  static Daemon* self = &d;
  signal(SIGTERM, [](int) {
    self->stop_spares();
    _exit(0);
  });
  metrics().describe("everserve_node_spare_starts_total", "Spares this daemon started (restarts included)", "counter");
  metrics().describe("everserve_node_processes_lost_total", "Engine processes the watcher found exiting", "counter");
  ES_INFO("node %s serving %s, coordinator %s", d.node.c_str(), socket.c_str(), d.coordinator.c_str());
  d.loop.run();
  return 0;
}
