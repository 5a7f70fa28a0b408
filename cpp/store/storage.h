// Storage of the per-node KV mirror: one engine's committed KV rows, per rank and table, in
// shared-memory files a restoring process maps directly.
//
// Layout: <data dir>/<engine>/rank<r>/table<t>.rows holds num_slots rows of row_bytes each (the
// row of a slot is its [2, head_dim] K/V pair for one layer and one kv head; table = layer * 1000 +
// head slot). Next to each table the store keeps, per slot, the step that last wrote it (0: never)
// and the row's CRC32C. A commit names one staging file the worker wrote in the same directory and
// where each table's rows start in it; the store copies the rows into the tables (runs of
// consecutive slots as one copy), stamps them, and records the request's committed token counts.
// A commit from an older epoch than the rank's is refused (a partitioned old member cannot write
// over the new one's rows). A restore names, per table, the slot ranges written since a step.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "everserve_pb.h"
#include "util.h"

namespace es {

struct Table {
  uint32_t id = 0;
  std::string dtype;
  std::vector<uint32_t> shape;
  size_t row_bytes = 0;
  std::unique_ptr<Mapping> rows;
  std::vector<uint64_t> written_step;
  std::vector<uint32_t> crc;
  size_t written = 0;
  std::vector<mirror::SlotRange> written_since(uint64_t since) const;
};

struct RankState {
  uint64_t epoch = 0, step = 0;
  uint64_t fence_epoch = 0;  // highest epoch a change told this store about
  bool caught_up = false;    // a replica that has every step of its source
  std::map<std::string, std::unique_ptr<Mapping>> stages;
  std::map<uint32_t, Table> tables;
  std::map<std::string, uint64_t> committed;
  std::vector<std::string> replicate_to;
};

struct EngineState {
  std::map<uint32_t, RankState> ranks;
  std::map<std::string, uint64_t> committed;  // every rank's requests (a request lives on all ranks)
};

size_t dtype_bytes(const std::string& dtype);

class Storage {
 public:
  Storage(std::string data_dir, size_t num_slots, size_t budget_bytes);
  std::string rank_dir(const std::string& engine, uint32_t rank) const;
  std::string open(const std::string& engine, uint32_t rank, std::string& stage_prefix, std::string& err);
  bool prepare(const mirror::Prepare& p, std::string& err);
  bool commit(const mirror::Commit& c, std::string& err);
  void restore(const mirror::RestoreRequest& r, mirror::RestoreReply& out) const;
  void evicted(const mirror::Evicted& e);
  void finished(const mirror::Finished& f);
  void committed(const mirror::CommittedQuery& q, mirror::CommittedReply& out) const;
  void rows(const mirror::RowsQuery& q, mirror::RowsReply& out) const;
  void state(const mirror::ReplicaStateQuery& q, mirror::ReplicaState& out) const;
  bool caught_up(const mirror::CaughtUp& c);
  // The rows a commit wrote, as replication messages of at most `max_bytes` each.
  std::vector<mirror::Replicated> replicated_of(const mirror::Commit& c, size_t max_bytes) const;
  bool apply_replicated(const mirror::Replicated& r, std::string& err);
  // Every written row of a rank (and its committed counts), as replication messages: what a new
  // replica needs before the rank's next commits reach it.
  std::vector<mirror::Replicated> snapshot_of(const std::string& engine, uint32_t rank, size_t max_bytes) const;
  void set_replicas(const std::string& engine, uint32_t rank, const std::vector<std::string>& targets);
  std::vector<std::string> replicas(const std::string& engine, uint32_t rank) const;
  size_t in_use() const { return in_use_; }
  size_t budget() const { return budget_; }
  size_t num_slots() const { return num_slots_; }

 private:
  Table* table_for(RankState& r, const std::string& dir, uint32_t id, const std::string& dtype,
                   const std::vector<uint32_t>& shape, std::string& err);
  std::string data_dir_;
  size_t num_slots_, budget_;
  size_t in_use_ = 0;
  uint64_t stage_seq_ = 0;
  std::map<std::string, EngineState> engines_;
};

}  // namespace es
