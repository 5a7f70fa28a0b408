// The node's compile cache: the built kernel artifacts a rank loads, moved between nodes by their
// stores so that a spare on a node without them can take a rank.
//
// Layout under the store's --compile-cache-dir: `<key>/<digest>/manifest.json` (key, digest and
// the files with their sizes and sha256) and `<key>/<digest>/files/<path>`. A serving worker
// publishes its artifacts there (everserve_b200.contract.compile_cache); a holder's store serves
// exactly the files its manifest lists, each checked against its sha256 as it is read, and only
// for the (key, digest) asked; a fetching store pulls them one chunk per request from the first
// holder that answers, checks each again, renames each into place and writes the manifest last,
// so a manifest present is the whole set in place.
//
// Reference parity: store/src/cache.rs (the same contract: manifest-listed files, per-file
// sha256, chunked reads, manifest written last) and the mirror.proto Cache* messages.
#pragma once

#include <mutex>
#include <string>

#include "everserve_pb.h"
#include "tls.h"

namespace es {

constexpr size_t kCacheChunkBytes = 4u << 20;

class CompileCacheDir {
 public:
  explicit CompileCacheDir(std::string dir) : dir_(std::move(dir)) {}
  bool enabled() const { return !dir_.empty(); }
  bool manifest(const std::string& key, const std::string& digest, mirror::CacheManifest& out,
                std::string& err) const;
  // Up to kCacheChunkBytes of a listed file from `offset` (empty at its end).
  bool read(const mirror::CacheRead& r, std::string& chunk, std::string& err) const;
  // Pull (key, digest) from the first holder (a store's replica address) that has it; a set
  // already in place is not fetched again. Blocking; run it off the loop.
  bool fetch(const mirror::CacheFetch& f, std::string& err);

 private:
  std::string base(const std::string& key, const std::string& digest) const;
  std::string dir_;
  std::mutex fetch_mu_;  // one fetch at a time: two asks for a set fetch it once
};

}  // namespace es
