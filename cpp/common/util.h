// Logging, CRC32C, a small JSON reader, file mapping and process helpers for the control plane.
#pragma once

#include <cstdint>
#include <cstdio>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace es {

// ---- logs: text by default, one JSON object per line when EVERSERVE_LOG_FORMAT=json ------------
void log_init(const char* component);
void logf(const char* level, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
#define ES_INFO(...) ::es::logf("info", __VA_ARGS__)
#define ES_WARN(...) ::es::logf("warn", __VA_ARGS__)
#define ES_ERROR(...) ::es::logf("error", __VA_ARGS__)

// ---- CRC32C (Castagnoli polynomial 0x82F63B78, reflected), table-driven ------------------------
uint32_t crc32c(const void* data, size_t n, uint32_t crc = 0);

// ---- JSON ----------------------------------------------------------------------------------------
struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const std::string& k) const;
  // A proto3 JSON field by its lowerCamelCase name, or by the proto field name it came from
  // ("outcomesInOrder" or "outcomes_in_order"): proto3 JSON readers accept both.
  const Json* field(const std::string& camel) const;
  static bool parse(const std::string& text, Json& out, std::string* err = nullptr);
  std::string dump() const;
};
std::string json_escape(const std::string& s);

// ---- files ---------------------------------------------------------------------------------------
// A shared file mapping (MAP_SHARED), created at `size` when `create`.
struct Mapping {
  void* addr = nullptr;
  size_t size = 0;
  std::string path;
  ~Mapping();
  static std::unique_ptr<Mapping> open(const std::string& path, size_t size, bool create, std::string* err = nullptr);
};
// Names of the entries of a directory (no "." or ".."); empty when it cannot be read.
std::vector<std::string> list_dir(const std::string& dir);
bool mkdirs(const std::string& path, int mode = 0770);
bool read_file(const std::string& path, std::string& out);
bool write_file_atomic(const std::string& path, const std::string& data);
std::string env_or(const char* name, const std::string& dflt);
// Run `argv` (PATH searched) and capture its standard output; false if it cannot start, exits
// non-zero, or runs past `timeout_ms` (then it is killed).
bool run_capture(const std::vector<std::string>& argv, int timeout_ms, std::string& out);
// Standard base64 (RFC 4648, padded); decode skips line breaks, false on another character.
std::string base64_encode(const std::string& in);
bool base64_decode(const std::string& in, std::string& out);

// ---- processes -----------------------------------------------------------------------------------
// /proc/<pid>/stat state: 'R','S','D','Z','X',... or 0 when the process does not exist.
char proc_state(int pid);

}  // namespace es
