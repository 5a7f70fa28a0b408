#include "cache.h"

#include <openssl/evp.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <fstream>
#include <memory>

#include "net.h"
#include "tls.h"
#include "util.h"

namespace es {

namespace {

struct Sha256 {
  EVP_MD_CTX* ctx = EVP_MD_CTX_new();
  Sha256() { EVP_DigestInit_ex(ctx, EVP_sha256(), nullptr); }
  ~Sha256() { EVP_MD_CTX_free(ctx); }
  void update(const char* p, size_t n) { EVP_DigestUpdate(ctx, p, n); }
  std::string hex() {
    unsigned char md[EVP_MAX_MD_SIZE];
    unsigned int n = 0;
    EVP_DigestFinal_ex(ctx, md, &n);
    static const char* d = "0123456789abcdef";
    std::string out;
    for (unsigned int i = 0; i < n; i++) {
      out.push_back(d[md[i] >> 4]);
      out.push_back(d[md[i] & 15]);
    }
    return out;
  }
};

// A key or digest names a directory: letters, digits, '.', '-', '_' only, not "." or "..".
bool safe_name(const std::string& s) {
  if (s.empty() || s == "." || s == ".." || s.size() > 200) return false;
  for (char c : s)
    if (!(isalnum((unsigned char)c) || c == '.' || c == '-' || c == '_')) return false;
  return true;
}

// A listed file's path: relative, no "..", no empty or "." components.
bool safe_path(const std::string& p) {
  if (p.empty() || p[0] == '/' || p.size() > 1024) return false;
  size_t a = 0;
  for (;;) {
    const size_t b = p.find('/', a);
    const std::string part = p.substr(a, b == std::string::npos ? std::string::npos : b - a);
    if (part.empty() || part == "." || part == "..") return false;
    if (b == std::string::npos) return true;
    a = b + 1;
  }
}

bool parse_manifest(const std::string& text, mirror::CacheManifest& m, std::string& err) {
  Json j;
  if (!Json::parse(text, j, &err) || j.kind != Json::Object) {
    if (err.empty()) err = "a manifest is a JSON object";
    return false;
  }
  if (const Json* k = j.get("key")) m.key = k->str;
  if (const Json* d = j.get("digest")) m.digest = d->str;
  if (const Json* fs = j.get("files"))
    for (auto& f : fs->arr) {
      mirror::CacheFile cf;
      if (const Json* p = f.get("path")) cf.path = p->str;
      if (const Json* s = f.get("size")) cf.size = s->kind == Json::Number ? (uint64_t)s->num : std::stoull(s->str);
      if (const Json* h = f.get("sha256")) cf.sha256 = h->str;
      if (!safe_path(cf.path)) {
        err = "a manifest lists an unsafe path: " + cf.path;
        return false;
      }
      m.files.push_back(cf);
    }
  return true;
}

std::string manifest_json(const mirror::CacheManifest& m) {
  std::string o = "{\"key\":\"" + json_escape(m.key) + "\",\"digest\":\"" + json_escape(m.digest) + "\",\"files\":[";
  for (size_t i = 0; i < m.files.size(); i++)
    o += std::string(i ? "," : "") + "{\"path\":\"" + json_escape(m.files[i].path) + "\",\"size\":" +
         std::to_string(m.files[i].size) + ",\"sha256\":\"" + json_escape(m.files[i].sha256) + "\"}";
  return o + "]}";
}

bool ask(tls::Stream& st, const mirror::MirrorRequest& req, mirror::MirrorReply& rep, int timeout_ms, std::string& err) {
  std::string frame;
  if (!st.write_frame(req.serialize(), timeout_ms) || !st.read_frame(frame, timeout_ms)) {
    err = "no answer";
    return false;
  }
  if (!rep.parse(frame)) {
    err = "malformed answer";
    return false;
  }
  if (!rep.error.empty()) {
    err = rep.error;
    return false;
  }
  return true;
}

}  // namespace

std::string CompileCacheDir::base(const std::string& key, const std::string& digest) const {
  return dir_ + "/" + key + "/" + digest;
}

bool CompileCacheDir::manifest(const std::string& key, const std::string& digest, mirror::CacheManifest& out,
                               std::string& err) const {
  if (!enabled()) {
    err = "this store keeps no compile caches (no --compile-cache-dir)";
    return false;
  }
  if (!safe_name(key) || !safe_name(digest)) {
    err = "a cache key and digest are plain names";
    return false;
  }
  std::string text;
  if (!read_file(base(key, digest) + "/manifest.json", text)) {
    err = "no compile cache " + key + "/" + digest + " here";
    return false;
  }
  out = mirror::CacheManifest{};
  if (!parse_manifest(text, out, err)) return false;
  if (out.key != key || out.digest != digest) {
    err = "the manifest held is of " + out.key + "/" + out.digest;
    return false;
  }
  return true;
}

bool CompileCacheDir::read(const mirror::CacheRead& r, std::string& chunk, std::string& err) const {
  mirror::CacheManifest m;
  if (!manifest(r.key, r.digest, m, err)) return false;
  const mirror::CacheFile* f = nullptr;
  for (auto& x : m.files)
    if (x.path == r.path) f = &x;
  if (f == nullptr) {
    err = r.path + " is not in the manifest";
    return false;
  }
  std::ifstream in(base(r.key, r.digest) + "/files/" + r.path, std::ios::binary);
  if (!in) {
    err = "cannot open " + r.path;
    return false;
  }
  if (r.offset >= f->size) {
    chunk.clear();
    return true;
  }
  in.seekg((std::streamoff)r.offset);
  const size_t n = (size_t)std::min<uint64_t>(kCacheChunkBytes, f->size - r.offset);
  chunk.resize(n);
  in.read(&chunk[0], (std::streamsize)n);
  chunk.resize((size_t)in.gcount());
  return true;
}

bool CompileCacheDir::fetch(const mirror::CacheFetch& f, std::string& err) {
  std::lock_guard<std::mutex> g(fetch_mu_);
  mirror::CacheManifest have;
  std::string ignored;
  if (manifest(f.key, f.digest, have, ignored)) return true;  // already in place
  if (!enabled()) {
    err = "this store keeps no compile caches (no --compile-cache-dir)";
    return false;
  }
  if (!safe_name(f.key) || !safe_name(f.digest)) {
    err = "a cache key and digest are plain names";
    return false;
  }
  if (f.holders.empty()) {
    err = "no holder named";
    return false;
  }
  std::string why;
  for (const auto& holder : f.holders) {
    Address a;
    tls::Stream st;
    std::string e;
    if (!Address::parse(holder, a) || !tls::connect_stream(a, 5000, st, &e)) {
      why += holder + ": unreachable; ";
      continue;
    }
    std::unique_ptr<tls::Stream, void (*)(tls::Stream*)> closer(&st, [](tls::Stream* s) { s->close(); });
    mirror::MirrorRequest q;
    q.has_cache_manifest = true;
    q.cache_manifest.key = f.key;
    q.cache_manifest.rank = f.rank;
    q.cache_manifest.dp = f.dp;
    q.cache_manifest.digest = f.digest;
    mirror::MirrorReply rep;
    if (!ask(st, q, rep, 30000, e) || !rep.has_cache_manifest) {
      why += holder + ": " + (e.empty() ? "no manifest" : e) + "; ";
      continue;
    }
    const mirror::CacheManifest m = rep.cache_manifest;
    if (m.key != f.key || m.digest != f.digest) {
      why += holder + ": answered another set; ";
      continue;
    }
    bool ok = true;
    const std::string root = base(f.key, f.digest);
    for (const auto& file : m.files) {
      if (!safe_path(file.path)) {
        why += holder + ": unsafe path " + file.path + "; ";
        ok = false;
        break;
      }
      const std::string dest = root + "/files/" + file.path;
      mkdirs(dest.substr(0, dest.rfind('/')));
      const std::string part = dest + ".part";
      std::ofstream out(part, std::ios::binary | std::ios::trunc);
      Sha256 h;
      uint64_t off = 0;
      while (ok && off < file.size) {
        mirror::MirrorRequest r;
        r.has_cache_read = true;
        r.cache_read.key = f.key;
        r.cache_read.rank = f.rank;
        r.cache_read.dp = f.dp;
        r.cache_read.digest = f.digest;
        r.cache_read.path = file.path;
        r.cache_read.offset = off;
        mirror::MirrorReply cr;
        if (!ask(st, r, cr, 30000, e) || !cr.has_cache_chunk || cr.cache_chunk.data.empty()) {
          why += holder + ": reading " + file.path + ": " + (e.empty() ? "short file" : e) + "; ";
          ok = false;
          break;
        }
        out.write(cr.cache_chunk.data.data(), (std::streamsize)cr.cache_chunk.data.size());
        h.update(cr.cache_chunk.data.data(), cr.cache_chunk.data.size());
        off += cr.cache_chunk.data.size();
      }
      out.close();
      if (ok && (off != file.size || h.hex() != file.sha256)) {
        why += holder + ": " + file.path + " does not match its sha256; ";
        ok = false;
      }
      if (!ok) {
        ::unlink(part.c_str());
        break;
      }
      ::chmod(part.c_str(), 0660);
      if (::rename(part.c_str(), dest.c_str()) != 0) {
        why += "cannot place " + file.path + "; ";
        ok = false;
        break;
      }
    }
    if (!ok) continue;
    if (!write_file_atomic(root + "/manifest.json", manifest_json(m))) {  // last: the set is in place
      why += "cannot write the manifest; ";
      continue;
    }
    return true;
  }
  err = "no holder served " + f.key + "/" + f.digest + ": " + why;
  return false;
}

}  // namespace es
