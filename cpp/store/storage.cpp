#include "storage.h"

#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>

namespace es {

// A fixed pool of commit workers (at most 8, one less than the cores). `parallel_for(n, fn)` runs
// fn(0..n-1) over the pool and the calling thread and returns when every call has finished; calls
// are serialised (the store's loop makes one at a time).
namespace {
class CommitPool {
 public:
  CommitPool() {
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const unsigned n = std::min(8u, hw > 1 ? hw - 1 : 0u);
    for (unsigned i = 0; i < n; i++) threads_.emplace_back([this] { loop(); });
  }
  ~CommitPool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : threads_) t.join();
  }
  void run(size_t n, const std::function<void(size_t)>& fn) {
    if (threads_.empty() || n < 2) {
      for (size_t i = 0; i < n; i++) fn(i);
      return;
    }
    std::unique_lock<std::mutex> g(mu_);
    fn_ = &fn;
    n_ = n;
    next_.store(0);
    busy_ = threads_.size();
    gen_++;
    g.unlock();
    cv_.notify_all();
    work();
    g.lock();
    done_cv_.wait(g, [this] { return busy_ == 0; });
    fn_ = nullptr;
  }

 private:
  void work() {
    for (size_t i = next_.fetch_add(1); i < n_; i = next_.fetch_add(1)) (*fn_)(i);
  }
  void loop() {
    uint64_t seen = 0;
    std::unique_lock<std::mutex> g(mu_);
    while (true) {
      cv_.wait(g, [&] { return stop_ || gen_ != seen; });
      if (stop_) return;
      seen = gen_;
      g.unlock();
      work();
      g.lock();
      if (--busy_ == 0) done_cv_.notify_all();
    }
  }
  std::vector<std::thread> threads_;
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(size_t)>* fn_ = nullptr;
  size_t n_ = 0;
  std::atomic<size_t> next_{0};
  size_t busy_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

void parallel_for(size_t n, const std::function<void(size_t)>& fn) {
  static CommitPool pool;
  pool.run(n, fn);
}
}  // namespace

size_t dtype_bytes(const std::string& d) {
  if (d == "float8_e4m3fn" || d == "float8_e5m2" || d == "int8" || d == "uint8") return 1;
  if (d == "float16" || d == "bfloat16" || d == "int16") return 2;
  if (d == "float32" || d == "int32") return 4;
  if (d == "float64" || d == "int64") return 8;
  return 0;
}

std::vector<mirror::SlotRange> Table::written_since(uint64_t since) const {
  std::vector<mirror::SlotRange> out;
  int64_t start = -1;
  for (size_t s = 0; s <= written_step.size(); s++) {
    const bool w = s < written_step.size() && written_step[s] != 0 && written_step[s] > since;
    if (w && start < 0) start = (int64_t)s;
    if (!w && start >= 0) {
      mirror::SlotRange r;
      r.start = start;
      r.count = (int64_t)s - start;
      out.push_back(r);
      start = -1;
    }
  }
  return out;
}

Storage::Storage(std::string data_dir, size_t num_slots, size_t budget_bytes)
    : data_dir_(std::move(data_dir)), num_slots_(num_slots), budget_(budget_bytes) {}

std::string Storage::rank_dir(const std::string& engine, uint32_t rank) const {
  return data_dir_ + "/" + engine + "/rank" + std::to_string(rank);
}

static bool safe_name(const std::string& s) {
  return !s.empty() && s.find('/') == std::string::npos && s != "." && s != "..";
}

std::string Storage::open(const std::string& engine, uint32_t rank, std::string& stage_prefix, std::string& err) {
  if (!safe_name(engine)) {
    err = "bad engine name";
    return "";
  }
  const std::string dir = rank_dir(engine, rank);
  if (!mkdirs(dir)) {
    err = "cannot create " + dir;
    return "";
  }
  engines_[engine].ranks[rank];
  stage_prefix = "stage" + std::to_string(getpid()) + "-" + std::to_string(++stage_seq_) + "-";
  return dir;
}

Table* Storage::table_for(RankState& r, const std::string& dir, uint32_t id, const std::string& dtype,
                          const std::vector<uint32_t>& shape, std::string& err) {
  auto it = r.tables.find(id);
  if (it != r.tables.end()) {
    if (it->second.dtype != dtype || it->second.shape != shape) {
      err = "table " + std::to_string(id) + ": row shape or dtype differs from the table's";
      return nullptr;
    }
    return &it->second;
  }
  const size_t eb = dtype_bytes(dtype);
  if (eb == 0) {
    err = "unknown dtype " + dtype;
    return nullptr;
  }
  size_t row = eb;
  for (auto d : shape) row *= d;
  const size_t bytes = row * num_slots_;
  if (in_use_ + bytes > budget_) {
    err = "budget: " + std::to_string(in_use_ + bytes) + " bytes needed, budget " + std::to_string(budget_);
    return nullptr;
  }
  Table t;
  t.id = id;
  t.dtype = dtype;
  t.shape = shape;
  t.row_bytes = row;
  t.rows = Mapping::open(dir + "/table" + std::to_string(id) + ".rows", bytes, true, &err);
  if (!t.rows) return nullptr;
  t.written_step.assign(num_slots_, 0);
  t.crc.assign(num_slots_, 0);
  in_use_ += bytes;
  auto res = r.tables.emplace(id, std::move(t));
  return &res.first->second;
}

bool Storage::prepare(const mirror::Prepare& p, std::string& err) {
  RankState& r = engines_[p.engine].ranks[p.rank];
  const std::string dir = rank_dir(p.engine, p.rank);
  mkdirs(dir);
  for (uint32_t id : p.tables) {
    Table* t = table_for(r, dir, id, p.dtype, p.shape, err);
    if (t == nullptr) return false;
    // touch every page now, so the first commit does not fault them in on the critical path
    auto* b = static_cast<volatile char*>(t->rows->addr);
    for (size_t off = 0; off < t->rows->size; off += 4096) b[off] = b[off];
  }
  return true;
}

bool Storage::commit(const mirror::Commit& c, std::string& err) {
  EngineState& eng = engines_[c.engine];
  RankState& r = eng.ranks[c.rank];
  if (c.epoch < r.epoch || c.epoch < r.fence_epoch) {
    err = "stale epoch " + std::to_string(c.epoch) + " (rank at " + std::to_string(r.epoch) + ")";
    return false;
  }
  if (c.has_staged) {
    const mirror::StagedStep& b = c.staged;
    if (!safe_name(b.stage)) {
      err = "bad stage name";
      return false;
    }
    const std::string dir = rank_dir(c.engine, c.rank);
    auto st = r.stages.find(b.stage);
    if (st == r.stages.end()) {
      auto m = Mapping::open(dir + "/" + b.stage, 0, false, &err);
      if (!m) return false;
      st = r.stages.emplace(b.stage, std::move(m)).first;
    }
    const char* stage = static_cast<const char*>(st->second->addr);
    const size_t stage_bytes = st->second->size;
    for (size_t s = 0; s < b.slots.size(); s++) {
      if (b.slots[s] >= (int64_t)num_slots_) {
        err = "slot " + std::to_string(b.slots[s]) + " outside the store's " + std::to_string(num_slots_);
        return false;
      }
    }
    // validate every table and the file length before writing anything
    std::vector<std::pair<Table*, uint64_t>> plan;
    for (size_t li = 0; li < b.layers.size(); li++) {
      for (size_t h = 0; h < b.heads.size(); h++) {
        const uint32_t id = b.layers[li] * b.table_stride + b.heads[h];
        const uint64_t off = b.base_offset + (uint64_t)b.layers[li] * b.layer_stride + (uint64_t)h * b.head_stride;
        Table* t = table_for(r, dir, id, b.dtype, b.shape, err);
        if (t == nullptr) return false;
        if (off + b.slots.size() * t->row_bytes > stage_bytes) {
          err = "staging file " + b.stage + " is shorter than the descriptor";
          return false;
        }
        plan.emplace_back(t, off);
      }
    }
    const uint64_t stamp = c.step == 0 ? 1 : c.step;
    // tables are independent: their copies and checksums run on the commit workers
    parallel_for(plan.size(), [&](size_t pi) {
      Table* t = plan[pi].first;
      const uint64_t off = plan[pi].second;
      char* rows = static_cast<char*>(t->rows->addr);
      for (size_t i = 0; i < b.slots.size();) {
        const int64_t s0 = b.slots[i];
        if (s0 < 0) {
          i++;
          continue;
        }
        size_t n = 1;
        while (i + n < b.slots.size() && b.slots[i + n] == s0 + (int64_t)n) n++;
        std::memcpy(rows + (size_t)s0 * t->row_bytes, stage + off + i * t->row_bytes, n * t->row_bytes);
        for (size_t k = 0; k < n; k++) {
          const size_t s = (size_t)s0 + k;
          if (t->written_step[s] == 0) t->written++;
          t->written_step[s] = stamp;
          t->crc[s] = crc32c(rows + s * t->row_bytes, t->row_bytes);
        }
        i += n;
      }
    });
  }
  r.epoch = c.epoch;
  r.step = c.step;
  for (size_t i = 0; i < c.request_ids.size() && i < c.committed_tokens.size(); i++) {
    r.committed[c.request_ids[i]] = c.committed_tokens[i];
    eng.committed[c.request_ids[i]] = c.committed_tokens[i];
  }
  return true;
}

void Storage::restore(const mirror::RestoreRequest& q, mirror::RestoreReply& out) const {
  auto e = engines_.find(q.engine);
  if (e == engines_.end()) return;
  auto r = e->second.ranks.find(q.rank);
  if (r == e->second.ranks.end()) return;
  const std::string dir = rank_dir(q.engine, q.rank);
  for (auto& [id, t] : r->second.tables) {
    mirror::TableRef ref;
    ref.layer = id;
    ref.path = dir + "/table" + std::to_string(id) + ".rows";
    ref.dtype = t.dtype;
    ref.shape = {(uint32_t)num_slots_};
    ref.shape.insert(ref.shape.end(), t.shape.begin(), t.shape.end());
    ref.written = t.written_since(q.since_step);
    out.tables.push_back(std::move(ref));
  }
  for (auto& [id, n] : r->second.committed) {
    out.request_ids.push_back(id);
    out.committed_tokens.push_back(n);
  }
  out.step = r->second.step;
}

void Storage::evicted(const mirror::Evicted& ev) {
  EngineState& eng = engines_[ev.engine];
  eng.committed[ev.request_id] = ev.kept_tokens;
  for (auto& [rank, r] : eng.ranks) {
    auto it = r.committed.find(ev.request_id);
    if (it != r.committed.end()) it->second = ev.kept_tokens;
  }
}

void Storage::finished(const mirror::Finished& f) {
  EngineState& eng = engines_[f.engine];
  for (const auto& id : f.request_ids) {
    eng.committed.erase(id);
    for (auto& [rank, r] : eng.ranks) r.committed.erase(id);
  }
}

void Storage::committed(const mirror::CommittedQuery& q, mirror::CommittedReply& out) const {
  auto e = engines_.find(q.engine);
  for (const auto& id : q.request_ids) {
    uint64_t n = 0;
    if (e != engines_.end()) {
      auto it = e->second.committed.find(id);
      if (it != e->second.committed.end()) n = it->second;
    }
    out.request_ids.push_back(id);
    out.committed_tokens.push_back(n);
  }
}

void Storage::rows(const mirror::RowsQuery& q, mirror::RowsReply& out) const {
  auto e = engines_.find(q.engine);
  if (e == engines_.end()) return;
  auto r = e->second.ranks.find(q.rank);
  if (r == e->second.ranks.end()) return;
  out.epoch = r->second.epoch;
  out.step = r->second.step;
  auto t = r->second.tables.find(q.table);
  if (t == r->second.tables.end()) return;
  const char* rows = static_cast<const char*>(t->second.rows->addr);
  for (int64_t s : q.slots) {
    if (s < 0 || s >= (int64_t)num_slots_) continue;
    mirror::SlotRow row;
    row.slot = s;
    row.written_step = t->second.written_step[(size_t)s];
    row.data.assign(rows + (size_t)s * t->second.row_bytes, t->second.row_bytes);
    row.crc32c = t->second.crc[(size_t)s];
    out.rows.push_back(std::move(row));
  }
}

void Storage::state(const mirror::ReplicaStateQuery& q, mirror::ReplicaState& out) const {
  auto e = engines_.find(q.engine);
  if (e == engines_.end()) return;
  auto r = e->second.ranks.find(q.rank);
  if (r == e->second.ranks.end()) return;
  out.epoch = r->second.epoch;
  out.step = r->second.step;
  out.held = !r->second.tables.empty();
  out.caught_up = r->second.caught_up;
  out.fence_epoch = r->second.fence_epoch;
}

bool Storage::caught_up(const mirror::CaughtUp& c) {
  RankState& r = engines_[c.engine].ranks[c.rank];
  if (c.epoch < r.epoch) return false;
  r.caught_up = true;
  return true;
}

std::vector<mirror::Replicated> Storage::replicated_of(const mirror::Commit& c, size_t max_bytes) const {
  std::vector<mirror::Replicated> out;
  auto e = engines_.find(c.engine);
  if (e == engines_.end()) return out;
  auto r = e->second.ranks.find(c.rank);
  if (r == e->second.ranks.end()) return out;
  auto fresh = [&]() {
    mirror::Replicated m;
    m.engine = c.engine;
    m.rank = c.rank;
    m.epoch = c.epoch;
    m.step = c.step;
    return m;
  };
  mirror::Replicated cur = fresh();
  cur.request_ids = c.request_ids;
  cur.committed_tokens = c.committed_tokens;
  size_t bytes = 0;
  if (c.has_staged) {
    const auto& b = c.staged;
    for (size_t li = 0; li < b.layers.size(); li++) {
      for (size_t h = 0; h < b.heads.size(); h++) {
        const uint32_t id = b.layers[li] * b.table_stride + b.heads[h];
        auto t = r->second.tables.find(id);
        if (t == r->second.tables.end()) continue;
        mirror::ReplicatedTable rt;
        rt.table = id;
        rt.dtype = t->second.dtype;
        rt.shape = t->second.shape;
        const char* rows = static_cast<const char*>(t->second.rows->addr);
        for (int64_t s : b.slots) {
          if (s < 0) continue;
          rt.slots.push_back(s);
          rt.data.append(rows + (size_t)s * t->second.row_bytes, t->second.row_bytes);
          rt.crc32c.push_back(t->second.crc[(size_t)s]);
        }
        if (bytes + rt.data.size() > max_bytes && !cur.tables.empty()) {
          out.push_back(std::move(cur));
          cur = fresh();
          bytes = 0;
        }
        bytes += rt.data.size();
        cur.tables.push_back(std::move(rt));
      }
    }
  }
  out.push_back(std::move(cur));
  return out;
}

std::vector<mirror::Replicated> Storage::snapshot_of(const std::string& engine, uint32_t rank,
                                                     size_t max_bytes) const {
  std::vector<mirror::Replicated> out;
  auto e = engines_.find(engine);
  if (e == engines_.end()) return out;
  auto r = e->second.ranks.find(rank);
  if (r == e->second.ranks.end()) return out;
  auto fresh = [&]() {
    mirror::Replicated m;
    m.engine = engine;
    m.rank = rank;
    m.epoch = r->second.epoch;
    m.step = r->second.step;
    return m;
  };
  mirror::Replicated cur = fresh();
  for (auto& [rid, n] : r->second.committed) {
    cur.request_ids.push_back(rid);
    cur.committed_tokens.push_back(n);
  }
  size_t bytes = 0;
  for (auto& [id, t] : r->second.tables) {
    mirror::ReplicatedTable rt;
    rt.table = id;
    rt.dtype = t.dtype;
    rt.shape = t.shape;
    const char* rows = static_cast<const char*>(t.rows->addr);
    for (size_t s = 0; s < t.written_step.size(); s++) {
      if (t.written_step[s] == 0) continue;
      if (bytes + rt.data.size() + t.row_bytes > max_bytes && (!cur.tables.empty() || !rt.slots.empty())) {
        if (!rt.slots.empty()) cur.tables.push_back(rt);
        out.push_back(std::move(cur));
        cur = fresh();
        bytes = 0;
        rt.slots.clear();
        rt.data.clear();
        rt.crc32c.clear();
      }
      rt.slots.push_back((int64_t)s);
      rt.data.append(rows + s * t.row_bytes, t.row_bytes);
      rt.crc32c.push_back(t.crc[s]);
    }
    bytes += rt.data.size();
    if (!rt.slots.empty()) cur.tables.push_back(std::move(rt));
  }
  out.push_back(std::move(cur));
  return out;
}

bool Storage::apply_replicated(const mirror::Replicated& m, std::string& err) {
  EngineState& eng = engines_[m.engine];
  RankState& r = eng.ranks[m.rank];
  if (m.epoch < r.epoch) {
    err = "stale epoch";
    return false;
  }
  const std::string dir = rank_dir(m.engine, m.rank);
  mkdirs(dir);
  // check every row before writing any (a bad part is refused whole)
  for (const auto& rt : m.tables) {
    const size_t eb = dtype_bytes(rt.dtype);
    size_t row = eb;
    for (auto d : rt.shape) row *= d;
    if (eb == 0 || rt.crc32c.size() != rt.slots.size() || rt.data.size() != row * rt.slots.size()) {
      err = "table " + std::to_string(rt.table) + ": rows and checksums do not match";
      return false;
    }
    for (size_t i = 0; i < rt.slots.size(); i++) {
      if (crc32c(rt.data.data() + i * row, row) != rt.crc32c[i]) {
        err = "table " + std::to_string(rt.table) + " slot " + std::to_string(rt.slots[i]) + ": checksum mismatch";
        return false;
      }
      if (rt.slots[i] < 0 || rt.slots[i] >= (int64_t)num_slots_) {
        err = "slot out of range";
        return false;
      }
    }
  }
  const uint64_t stamp = m.step == 0 ? 1 : m.step;
  for (const auto& rt : m.tables) {
    Table* t = table_for(r, dir, rt.table, rt.dtype, rt.shape, err);
    if (t == nullptr) return false;
    char* rows = static_cast<char*>(t->rows->addr);
    for (size_t i = 0; i < rt.slots.size(); i++) {
      const size_t s = (size_t)rt.slots[i];
      std::memcpy(rows + s * t->row_bytes, rt.data.data() + i * t->row_bytes, t->row_bytes);
      if (t->written_step[s] == 0) t->written++;
      t->written_step[s] = stamp;
      t->crc[s] = rt.crc32c[i];
    }
  }
  r.epoch = m.epoch;
  r.step = std::max(r.step, m.step);
  for (size_t i = 0; i < m.request_ids.size() && i < m.committed_tokens.size(); i++) {
    r.committed[m.request_ids[i]] = m.committed_tokens[i];
    eng.committed[m.request_ids[i]] = m.committed_tokens[i];
  }
  return true;
}

void Storage::set_replicas(const std::string& engine, uint32_t rank, const std::vector<std::string>& targets) {
  engines_[engine].ranks[rank].replicate_to = targets;
}

std::vector<std::string> Storage::replicas(const std::string& engine, uint32_t rank) const {
  auto e = engines_.find(engine);
  if (e == engines_.end()) return {};
  auto r = e->second.ranks.find(rank);
  return r == e->second.ranks.end() ? std::vector<std::string>{} : r->second.replicate_to;
}

}  // namespace es
