#include <algorithm>
#include <dirent.h>
#include "util.h"

#include <errno.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <poll.h>
#include <signal.h>
#include <sys/stat.h>
#include <sys/wait.h>
#include <unistd.h>

#include <cmath>
#include <cstdarg>
#include <cstring>
#include <ctime>

#include "net.h"

namespace es {

static std::string g_component = "everserve";
static bool g_json = false;

void log_init(const char* component) {
  g_component = component;
  const char* f = getenv("EVERSERVE_LOG_FORMAT");
  g_json = f != nullptr && std::string(f) == "json";
}

void logf(const char* level, const char* fmt, ...) {
  char msg[4096];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof(msg), fmt, ap);
  va_end(ap);
  const uint64_t ms = now_ms();
  if (g_json) {
    fprintf(stderr, "{\"ts_ms\":%llu,\"level\":\"%s\",\"component\":\"%s\",\"msg\":\"%s\"}\n", (unsigned long long)ms,
            level, g_component.c_str(), json_escape(msg).c_str());
  } else {
    time_t t = (time_t)(ms / 1000);
    struct tm tmv;
    gmtime_r(&t, &tmv);
    char ts[32];
    strftime(ts, sizeof(ts), "%H:%M:%S", &tmv);
    fprintf(stderr, "%s.%03u %s %s: %s\n", ts, (unsigned)(ms % 1000), level, g_component.c_str(), msg);
  }
  fflush(stderr);
}

static uint32_t g_crc_table[256];
static bool g_crc_init = [] {
  for (uint32_t i = 0; i < 256; i++) {
    uint32_t c = i;
    for (int k = 0; k < 8; k++) c = (c & 1) ? (c >> 1) ^ 0x82F63B78u : c >> 1;
    g_crc_table[i] = c;
  }
  return true;
}();

static uint32_t crc32c_table(const uint8_t* p, size_t n, uint32_t crc) {
  (void)g_crc_init;
  for (size_t i = 0; i < n; i++) crc = g_crc_table[(crc ^ p[i]) & 0xFF] ^ (crc >> 8);
  return crc;
}

#if defined(__x86_64__)
// The same polynomial through the SSE4.2 crc32 instruction, eight bytes at a time (about an order
// of magnitude faster than the table: the store checksums every row it is sent).
__attribute__((target("sse4.2"))) static uint32_t crc32c_hw(const uint8_t* p, size_t n, uint32_t crc) {
  uint64_t c = crc;
  while (n >= 8) {
    uint64_t v;
    memcpy(&v, p, 8);
    c = __builtin_ia32_crc32di(c, v);
    p += 8;
    n -= 8;
  }
  uint32_t c32 = (uint32_t)c;
  while (n > 0) {
    c32 = __builtin_ia32_crc32qi(c32, *p++);
    n--;
  }
  return c32;
}
static const bool g_crc_hw = __builtin_cpu_supports("sse4.2");
#endif

uint32_t crc32c(const void* data, size_t n, uint32_t crc) {
  const auto* p = static_cast<const uint8_t*>(data);
#if defined(__x86_64__)
  if (g_crc_hw) return ~crc32c_hw(p, n, ~crc);
#endif
  return ~crc32c_table(p, n, ~crc);
}

// ---- JSON ----------------------------------------------------------------------------------------
namespace {
struct JP {
  const std::string& s;
  size_t i = 0;
  std::string err;
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\t' || s[i] == '\r')) i++;
  }
  bool fail(const char* m) {
    if (err.empty()) err = std::string(m) + " at " + std::to_string(i);
    return false;
  }
  bool str(std::string& out) {
    if (i >= s.size() || s[i] != '"') return fail("expected string");
    i++;
    while (i < s.size() && s[i] != '"') {
      char c = s[i++];
      if (c == '\\') {
        if (i >= s.size()) return fail("bad escape");
        char e = s[i++];
        switch (e) {
          case 'n': out.push_back('\n'); break;
          case 't': out.push_back('\t'); break;
          case 'r': out.push_back('\r'); break;
          case 'b': out.push_back('\b'); break;
          case 'f': out.push_back('\f'); break;
          case 'u': {
            if (i + 4 > s.size()) return fail("bad unicode escape");
            unsigned cp = (unsigned)strtoul(s.substr(i, 4).c_str(), nullptr, 16);
            i += 4;
            if (cp < 0x80) out.push_back((char)cp);
            else if (cp < 0x800) {
              out.push_back((char)(0xC0 | (cp >> 6)));
              out.push_back((char)(0x80 | (cp & 0x3F)));
            } else {
              out.push_back((char)(0xE0 | (cp >> 12)));
              out.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
              out.push_back((char)(0x80 | (cp & 0x3F)));
            }
            break;
          }
          default: out.push_back(e);
        }
      } else {
        out.push_back(c);
      }
    }
    if (i >= s.size()) return fail("unterminated string");
    i++;
    return true;
  }
  bool value(Json& v) {
    ws();
    if (i >= s.size()) return fail("unexpected end");
    const char c = s[i];
    if (c == '{') {
      v.kind = Json::Object;
      i++;
      ws();
      if (i < s.size() && s[i] == '}') {
        i++;
        return true;
      }
      while (true) {
        ws();
        std::string k;
        if (!str(k)) return false;
        ws();
        if (i >= s.size() || s[i] != ':') return fail("expected ':'");
        i++;
        Json child;
        if (!value(child)) return false;
        v.obj.emplace_back(std::move(k), std::move(child));
        ws();
        if (i < s.size() && s[i] == ',') {
          i++;
          continue;
        }
        if (i < s.size() && s[i] == '}') {
          i++;
          return true;
        }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = Json::Array;
      i++;
      ws();
      if (i < s.size() && s[i] == ']') {
        i++;
        return true;
      }
      while (true) {
        Json child;
        if (!value(child)) return false;
        v.arr.push_back(std::move(child));
        ws();
        if (i < s.size() && s[i] == ',') {
          i++;
          continue;
        }
        if (i < s.size() && s[i] == ']') {
          i++;
          return true;
        }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = Json::String;
      return str(v.str);
    }
    if (s.compare(i, 4, "true") == 0) {
      v.kind = Json::Bool;
      v.b = true;
      i += 4;
      return true;
    }
    if (s.compare(i, 5, "false") == 0) {
      v.kind = Json::Bool;
      i += 5;
      return true;
    }
    if (s.compare(i, 4, "null") == 0) {
      i += 4;
      return true;
    }
    char* end = nullptr;
    v.num = strtod(s.c_str() + i, &end);
    if (end == s.c_str() + i) return fail("bad value");
    v.kind = Json::Number;
    i = size_t(end - s.c_str());
    return true;
  }
};
}  // namespace

const Json* Json::get(const std::string& k) const {
  for (auto& kv : obj)
    if (kv.first == k) return &kv.second;
  return nullptr;
}

const Json* Json::field(const std::string& camel) const {
  if (const Json* v = get(camel)) return v;
  std::string snake;
  for (char c : camel) {
    if (c >= 'A' && c <= 'Z') {
      snake.push_back('_');
      snake.push_back((char)(c - 'A' + 'a'));
    } else {
      snake.push_back(c);
    }
  }
  return snake == camel ? nullptr : get(snake);
}

bool Json::parse(const std::string& text, Json& out, std::string* err) {
  JP p{text, 0, {}};
  if (!p.value(out)) {
    if (err) *err = p.err;
    return false;
  }
  return true;
}

std::string json_escape(const std::string& s) {
  std::string o;
  for (char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\t': o += "\\t"; break;
      case '\r': o += "\\r"; break;
      default:
        if ((unsigned char)c < 0x20) {
          char b[8];
          snprintf(b, sizeof(b), "\\u%04x", (unsigned char)c);
          o += b;
        } else {
          o.push_back(c);
        }
    }
  }
  return o;
}

std::string Json::dump() const {
  switch (kind) {
    case Null: return "null";
    case Bool: return b ? "true" : "false";
    case Number: {
      char buf[64];
      if (std::floor(num) == num && std::fabs(num) < 1e15) snprintf(buf, sizeof(buf), "%.0f", num);
      else snprintf(buf, sizeof(buf), "%.17g", num);
      return buf;
    }
    case String: return "\"" + json_escape(str) + "\"";
    case Array: {
      std::string o = "[";
      for (size_t i = 0; i < arr.size(); i++) o += (i ? "," : "") + arr[i].dump();
      return o + "]";
    }
    case Object: {
      std::string o = "{";
      for (size_t i = 0; i < obj.size(); i++) o += (i ? "," : "") + ("\"" + json_escape(obj[i].first) + "\":") + obj[i].second.dump();
      return o + "}";
    }
  }
  return "null";
}

// ---- files ---------------------------------------------------------------------------------------
Mapping::~Mapping() {
  if (addr != nullptr && addr != MAP_FAILED) munmap(addr, size);
}

std::unique_ptr<Mapping> Mapping::open(const std::string& path, size_t size, bool create, std::string* err) {
  const int fd = ::open(path.c_str(), create ? (O_RDWR | O_CREAT) : O_RDWR, 0660);
  if (fd < 0) {
    if (err) *err = "open " + path + ": " + strerror(errno);
    return nullptr;
  }
  struct stat st;
  fstat(fd, &st);
  if (create && (size_t)st.st_size < size && ftruncate(fd, (off_t)size) != 0) {
    if (err) *err = "ftruncate " + path + ": " + strerror(errno);
    ::close(fd);
    return nullptr;
  }
  if (!create) {
    if (size == 0) size = (size_t)st.st_size;
    if ((size_t)st.st_size < size) {
      if (err) *err = path + " is shorter than expected";
      ::close(fd);
      return nullptr;
    }
  }
  auto m = std::make_unique<Mapping>();
  m->size = size;
  m->path = path;
  m->addr = size ? mmap(nullptr, size, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0) : nullptr;
  ::close(fd);
  if (m->addr == MAP_FAILED) {
    m->addr = nullptr;
    if (err) *err = "mmap " + path + ": " + strerror(errno);
    return nullptr;
  }
  return m;
}

std::vector<std::string> list_dir(const std::string& dir) {
  std::vector<std::string> out;
  DIR* d = ::opendir(dir.c_str());
  if (!d) return out;
  while (dirent* e = ::readdir(d)) {
    const std::string n = e->d_name;
    if (n != "." && n != "..") out.push_back(n);
  }
  ::closedir(d);
  std::sort(out.begin(), out.end());
  return out;
}

bool mkdirs(const std::string& path, int mode) {
  std::string cur;
  for (size_t i = 0; i < path.size(); i++) {
    cur.push_back(path[i]);
    if ((path[i] == '/' && i > 0) || i + 1 == path.size()) {
      if (::mkdir(cur.c_str(), (mode_t)mode) != 0 && errno != EEXIST) return false;
    }
  }
  return true;
}

bool read_file(const std::string& path, std::string& out) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  char buf[65536];
  size_t n;
  out.clear();
  while ((n = fread(buf, 1, sizeof(buf), f)) > 0) out.append(buf, n);
  fclose(f);
  return true;
}

bool write_file_atomic(const std::string& path, const std::string& data) {
  const std::string tmp = path + ".tmp";
  FILE* f = fopen(tmp.c_str(), "wb");
  if (!f) return false;
  const bool ok = fwrite(data.data(), 1, data.size(), f) == data.size();
  fflush(f);
  fsync(fileno(f));
  fclose(f);
  return ok && rename(tmp.c_str(), path.c_str()) == 0;
}

std::string env_or(const char* name, const std::string& dflt) {
  const char* v = getenv(name);
  return v ? std::string(v) : dflt;
}

char proc_state(int pid) {
  std::string s;
  if (!read_file("/proc/" + std::to_string(pid) + "/stat", s)) return 0;
  const auto rp = s.rfind(')');
  if (rp == std::string::npos || rp + 2 >= s.size()) return 0;
  return s[rp + 2];
}

}  // namespace es

namespace es {

bool run_capture(const std::vector<std::string>& argv, int timeout_ms, std::string& out) {
  if (argv.empty()) return false;
  int fds[2];
  if (pipe2(fds, O_CLOEXEC) != 0) return false;
  const pid_t pid = fork();
  if (pid < 0) {
    ::close(fds[0]);
    ::close(fds[1]);
    return false;
  }
  if (pid == 0) {
    dup2(fds[1], 1);
    const int devnull = open("/dev/null", O_WRONLY);
    if (devnull >= 0) dup2(devnull, 2);
    std::vector<char*> a;
    for (auto& s : argv) a.push_back(const_cast<char*>(s.c_str()));
    a.push_back(nullptr);
    execvp(a[0], a.data());
    _exit(127);
  }
  ::close(fds[1]);
  out.clear();
  const uint64_t deadline = now_ms() + (uint64_t)timeout_ms;
  bool timed_out = false;
  char buf[4096];
  for (;;) {
    const int64_t left = (int64_t)deadline - (int64_t)now_ms();
    if (left <= 0) {
      timed_out = true;
      break;
    }
    pollfd p{fds[0], POLLIN, 0};
    const int r = poll(&p, 1, (int)left);
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) continue;
    const ssize_t n = ::read(fds[0], buf, sizeof buf);
    if (n < 0 && errno == EINTR) continue;
    if (n <= 0) break;
    out.append(buf, (size_t)n);
  }
  ::close(fds[0]);
  if (timed_out) kill(pid, SIGKILL);
  int status = 0;
  while (waitpid(pid, &status, 0) < 0 && errno == EINTR) {
  }
  return !timed_out && WIFEXITED(status) && WEXITSTATUS(status) == 0;
}

}  // namespace es

namespace es {

static const char* kB64 = "ABCDEFGHIJKLMNOPQRSTUVWXYZabcdefghijklmnopqrstuvwxyz0123456789+/";

std::string base64_encode(const std::string& in) {
  std::string out;
  size_t i = 0;
  for (; i + 2 < in.size(); i += 3) {
    const uint32_t v = ((uint8_t)in[i] << 16) | ((uint8_t)in[i + 1] << 8) | (uint8_t)in[i + 2];
    for (int s = 18; s >= 0; s -= 6) out.push_back(kB64[(v >> s) & 63]);
  }
  if (i + 1 == in.size()) {
    const uint32_t v = (uint8_t)in[i] << 16;
    out += {kB64[(v >> 18) & 63], kB64[(v >> 12) & 63], '=', '='};
  } else if (i + 2 == in.size()) {
    const uint32_t v = ((uint8_t)in[i] << 16) | ((uint8_t)in[i + 1] << 8);
    out += {kB64[(v >> 18) & 63], kB64[(v >> 12) & 63], kB64[(v >> 6) & 63], '='};
  }
  return out;
}

bool base64_decode(const std::string& in, std::string& out) {
  int val[256];
  for (int& v : val) v = -1;
  for (int k = 0; k < 64; k++) val[(uint8_t)kB64[k]] = k;
  out.clear();
  uint32_t acc = 0;
  int bits = 0;
  for (char c : in) {
    if (c == '=' || c == '\n' || c == '\r') continue;
    if (val[(uint8_t)c] < 0) return false;
    acc = (acc << 6) | (uint32_t)val[(uint8_t)c];
    bits += 6;
    if (bits >= 8) {
      bits -= 8;
      out.push_back((char)((acc >> bits) & 0xff));
    }
  }
  return true;
}

}  // namespace es
