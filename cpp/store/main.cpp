// everserve-store: the per-node KV mirror (one per node).
//
//   everserve-store --socket unix:/run/everserve/mirror.sock --data-dir /dev/shm/everserve/store
//                   [--slots N] [--budget-bytes B] [--replica-listen host:port]
//                   [--metrics-addr host:port] [--replication-queue-bytes Q] [--compile-cache-dir DIR]
// Every flag also reads an EVERSERVE_STORE_* environment variable.
//
// Workers speak mirror.proto over the Unix socket (Open, Prepare, Commit, Restore, Evicted,
// Finished, Committed, Rows, ReplicaState, CaughtUp, Replicate). Stores speak the same protocol to
// each other over TCP: after a commit of a rank that has replication targets, a carrier sends the
// step's rows (with their CRC32C) as Replicated messages of at most one frame each; the receiving
// store checks every checksum before it writes anything. The carrier's byte queue is bounded: a
// step that does not fit is dropped and counted, and the target re-syncs from a later snapshot.
#include <signal.h>
#include <unistd.h>

#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <mutex>
#include <thread>

#include "cache.h"
#include "everserve_pb.h"
#include "net.h"
#include "storage.h"
#include "telemetry.h"
#include "tls.h"
#include "util.h"

using namespace es;

namespace {

struct Options {
  std::string socket = "unix:/tmp/everserve-store.sock";
  std::string data_dir = "/dev/shm/everserve-store";
  size_t slots = 1 << 20;
  size_t budget = size_t(64) << 30;
  std::string replica_listen;
  std::string cache_dir;  // the node's compile cache ("" keeps none)
  std::string metrics_addr;
  size_t queue_bytes = size_t(1) << 30;
};

// One outgoing replication link per target address, with a bounded byte queue.
class Carrier {
 public:
  explicit Carrier(size_t cap) : cap_(cap) { th_ = std::thread([this] { run(); }); }
  void push(const std::string& target, std::string frame) {
    std::lock_guard<std::mutex> g(mu_);
    if (bytes_ + frame.size() > cap_) {
      metrics().inc("everserve_store_replication_dropped_total");
      return;
    }
    bytes_ += frame.size();
    q_.emplace_back(target, std::move(frame));
    cv_.notify_one();
  }

 private:
  void run() {
    std::map<std::string, tls::Stream> links;  // TLS when configured (the targets are TCP)
    while (true) {
      std::pair<std::string, std::string> item;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return !q_.empty(); });
        item = std::move(q_.front());
        q_.pop_front();
        bytes_ -= item.second.size();
      }
      for (int attempt = 0; attempt < 2; attempt++) {
        tls::Stream& st = links[item.first];
        if (st.fd < 0) {
          Address a;
          std::string err;
          if (!Address::parse(item.first, a) || !tls::connect_stream(a, 2000, st, &err)) {
            metrics().inc("everserve_store_replication_link_failures_total");
            break;
          }
        }
        std::string reply;
        if (st.write_frame(item.second, 10000) && st.read_frame(reply, 10000)) {
          mirror::MirrorReply r;
          if (r.parse(reply) && r.error.empty()) metrics().inc("everserve_store_replicated_total");
          else metrics().inc("everserve_store_replication_link_failures_total");
          break;
        }
        st.close();
      }
    }
  }
  size_t cap_;
  size_t bytes_ = 0;
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<std::pair<std::string, std::string>> q_;
  std::thread th_;
};

void handle(Storage& st, Carrier& carrier, CompileCacheDir& cache, Loop& loop, Conn& c, const std::string& frame) {
  mirror::MirrorRequest req;
  mirror::MirrorReply rep;
  if (!req.parse(frame)) {
    rep.error = "malformed request";
    loop.send(c.id, rep.serialize());
    return;
  }
  std::string err;
  const uint64_t t0 = now_us();
  if (req.has_open) {
    std::string prefix;
    const std::string dir = st.open(req.open.engine, req.open.rank, prefix, err);
    if (req.open.protocol != 0 && req.open.protocol < signals::ProtocolOldest_PROTOCOL_OLDEST) err = "protocol too old";
    if (err.empty()) {
      rep.has_opened = true;
      rep.opened.rank_dir = dir;
      rep.opened.stage_prefix = prefix;
    }
  } else if (req.has_prepare) {
    if (st.prepare(req.prepare, err)) rep.has_done = true;
  } else if (req.has_commit) {
    if (st.commit(req.commit, err)) {
      rep.has_commit_ack = true;
      rep.commit_ack.step = req.commit.step;
      metrics().inc("everserve_store_commits_total");
      for (const auto& target : st.replicas(req.commit.engine, req.commit.rank)) {
        for (auto& part : st.replicated_of(req.commit, kMaxFrame - 4096)) {
          mirror::MirrorRequest out;
          out.has_replicated = true;
          out.replicated = std::move(part);
          carrier.push(target, out.serialize());
        }
      }
    } else {
      metrics().inc("everserve_store_refusals_total");
    }
    metrics().set("everserve_store_bytes_in_use", {}, (double)st.in_use());
  } else if (req.has_restore) {
    rep.has_restore = true;
    st.restore(req.restore, rep.restore);
    size_t rows = 0;
    for (auto& t : rep.restore.tables)
      for (auto& r : t.written) rows += (size_t)r.count;
    metrics().inc("everserve_store_restore_rows_total", {}, (double)rows);
    metrics().observe("everserve_store_restore_seconds", {}, (now_us() - t0) * 1e-6);
  } else if (req.has_committed) {
    rep.has_committed = true;
    st.committed(req.committed, rep.committed);
  } else if (req.has_evicted) {
    st.evicted(req.evicted);
    rep.has_done = true;
  } else if (req.has_finished) {
    st.finished(req.finished);
    rep.has_done = true;
  } else if (req.has_rows) {
    rep.has_rows = true;
    st.rows(req.rows, rep.rows);
  } else if (req.has_replica_state) {
    rep.has_replica_state = true;
    st.state(req.replica_state, rep.replica_state);
  } else if (req.has_caught_up) {
    if (st.caught_up(req.caught_up)) rep.has_done = true;
    else err = "stale epoch";
  } else if (req.has_replicate) {
    const auto before = st.replicas(req.replicate.engine, req.replicate.rank);
    st.set_replicas(req.replicate.engine, req.replicate.rank, req.replicate.targets);
    // a new target first gets everything the rank has written (queued ahead of its next commits)
    for (const auto& target : req.replicate.targets) {
      if (std::find(before.begin(), before.end(), target) != before.end()) continue;
      metrics().inc("everserve_store_snapshots_total");
      for (auto& part : st.snapshot_of(req.replicate.engine, req.replicate.rank, kMaxFrame - 4096)) {
        mirror::MirrorRequest out;
        out.has_replicated = true;
        out.replicated = std::move(part);
        carrier.push(target, out.serialize());
      }
    }
    rep.has_done = true;
  } else if (req.has_replicated) {
    if (st.apply_replicated(req.replicated, err)) {
      rep.has_done = true;
      metrics().inc("everserve_store_replica_applied_total");
    } else {
      metrics().inc("everserve_store_refusals_total");
    }
  } else if (req.has_expect) {
    rep.has_done = true;
  } else if (req.has_cache_manifest) {
    if (cache.manifest(req.cache_manifest.key, req.cache_manifest.digest, rep.cache_manifest, err))
      rep.has_cache_manifest = true;
  } else if (req.has_cache_read) {
    if (cache.read(req.cache_read, rep.cache_chunk.data, err)) rep.has_cache_chunk = true;
  } else if (req.has_cache_fetch) {
    // pulled from the holders on a thread of its own; the answer comes when the set is in place
    const uint64_t conn = c.id;
    const mirror::CacheFetch f = req.cache_fetch;
    std::thread([&cache, &loop, conn, f] {
      std::string e;
      const uint64_t t = now_us();
      const bool ok = cache.fetch(f, e);
      metrics().inc("everserve_store_cache_fetches_total", {{"verdict", ok ? "ok" : "failed"}});
      if (ok) metrics().observe("everserve_store_cache_fetch_seconds", {}, (now_us() - t) * 1e-6);
      else ES_WARN("compile cache %s/%s: %s", f.key.c_str(), f.digest.c_str(), e.c_str());
      loop.post([&loop, conn, ok, e] {
        mirror::MirrorReply r;
        if (ok) r.has_done = true;
        r.error = ok ? "" : e;
        loop.send(conn, r.serialize());
      });
    }).detach();
    return;
  } else {
    err = "unsupported request";
  }
  rep.error = err;
  loop.send(c.id, rep.serialize());
}

}  // namespace

int main(int argc, char** argv) {
  {
    std::string terr;
    if (!es::tls::configure_from_env(&terr)) {
      fprintf(stderr, "TLS: %s\n", terr.c_str());
      return 2;
    }
  }
  log_init("store");
  signal(SIGPIPE, SIG_IGN);
  Options o;
  o.socket = env_or("EVERSERVE_STORE_SOCKET", o.socket);
  o.data_dir = env_or("EVERSERVE_STORE_DATA_DIR", o.data_dir);
  o.slots = std::stoull(env_or("EVERSERVE_STORE_SLOTS", std::to_string(o.slots)));
  o.budget = std::stoull(env_or("EVERSERVE_STORE_BUDGET_BYTES", std::to_string(o.budget)));
  o.replica_listen = env_or("EVERSERVE_STORE_REPLICA_LISTEN", "");
  o.metrics_addr = env_or("EVERSERVE_METRICS_ADDR", "");
  o.queue_bytes = std::stoull(env_or("EVERSERVE_STORE_REPLICATION_QUEUE_BYTES", std::to_string(o.queue_bytes)));
  o.cache_dir = env_or("EVERSERVE_STORE_COMPILE_CACHE_DIR", "");
  for (int i = 1; i + 1 < argc; i += 2) {
    const std::string k = argv[i], v = argv[i + 1];
    if (k == "--socket") o.socket = v;
    else if (k == "--data-dir") o.data_dir = v;
    else if (k == "--slots") o.slots = std::stoull(v);
    else if (k == "--budget-bytes") o.budget = std::stoull(v);
    else if (k == "--replica-listen") o.replica_listen = v;
    else if (k == "--metrics-addr") o.metrics_addr = v;
    else if (k == "--replication-queue-bytes") o.queue_bytes = std::stoull(v);
    else if (k == "--compile-cache-dir") o.cache_dir = v;
    else {
      fprintf(stderr, "unknown flag %s\n", k.c_str());
      return 2;
    }
  }
  metrics().describe("everserve_store_commits_total", "Commits accepted", "counter");
  metrics().describe("everserve_store_refusals_total", "Requests refused (stale epoch, budget, shape, checksum)", "counter");
  metrics().describe("everserve_store_bytes_in_use", "Bytes of table files held", "gauge");
  metrics().describe("everserve_store_restore_rows_total", "Rows named by restores", "counter");
  metrics().describe("everserve_store_restore_seconds", "Time to answer a restore", "histogram");
  metrics().describe("everserve_store_replicated_total", "Replication parts a target acknowledged", "counter");
  metrics().describe("everserve_store_replication_dropped_total", "Replication parts dropped by the bounded queue", "counter");
  metrics().describe("everserve_store_replication_link_failures_total", "Failed sends to a replication target", "counter");
  metrics().describe("everserve_store_snapshots_total", "Snapshots of a rank's rows sent to a new replication target", "counter");
  metrics().describe("everserve_store_cache_fetches_total", "Compile-cache fetches from holder stores, by verdict", "counter");
  metrics().describe("everserve_store_cache_fetch_seconds", "Time to put a compile cache in place", "histogram");
  metrics().describe("everserve_store_replica_applied_total", "Replication parts applied from a source store", "counter");
  mkdirs(o.data_dir);
  Storage st(o.data_dir, o.slots, o.budget);
  Carrier carrier(o.queue_bytes);
  CompileCacheDir cache(o.cache_dir);
  if (cache.enabled()) mkdirs(o.cache_dir);
  Loop loop;
  Address a;
  std::string err;
  if (!Address::parse(o.socket, a) || !loop.listen(a, [&](Conn& c) {
        c.on_frame = [&](Conn& cc, const std::string& f) { handle(st, carrier, cache, loop, cc, f); };
      }, &err)) {
    ES_ERROR("listen %s: %s", o.socket.c_str(), err.c_str());
    return 1;
  }
  if (!o.replica_listen.empty()) {
    Address ra;
    if (!Address::parse(o.replica_listen, ra) || !loop.listen(ra, [&](Conn& c) {
          c.on_frame = [&](Conn& cc, const std::string& f) { handle(st, carrier, cache, loop, cc, f); };
        }, &err)) {
      ES_ERROR("replica listen %s: %s", o.replica_listen.c_str(), err.c_str());
      return 1;
    }
  }
  if (!o.metrics_addr.empty() && !serve_http(loop, o.metrics_addr, nullptr, &err)) {
    ES_ERROR("metrics %s: %s", o.metrics_addr.c_str(), err.c_str());
    return 1;
  }
  loop.every(tls::reload_period_ms(), [] {  // renewed certificates, taken without a restart
    std::string terr;
    if (!tls::reload_if_changed(&terr)) ES_WARN("TLS reload: %s", terr.c_str());
  });
  ES_INFO("serving %s (data %s, %zu slots, budget %zu bytes)", o.socket.c_str(), o.data_dir.c_str(), o.slots, o.budget);
  loop.run();
  return 0;
}
