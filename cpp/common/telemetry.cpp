#include "telemetry.h"

#include <fcntl.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cctype>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <thread>

#include "net.h"
#include "tls.h"

namespace es {

static const double kBuckets[] = {0.0005, 0.001, 0.0025, 0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1, 2.5, 5, 10, 30};
constexpr int kNBuckets = sizeof(kBuckets) / sizeof(kBuckets[0]);

Registry& metrics() {
  static Registry r;
  return r;
}

std::string Registry::key(const Labels& l) {
  std::string k;
  for (size_t i = 0; i < l.size(); i++) {
    k += (i ? "," : "") + l[i].first + "=\"";
    for (char c : l[i].second) {
      if (c == '"' || c == '\\') k.push_back('\\');
      k.push_back(c == '\n' ? ' ' : c);
    }
    k += "\"";
  }
  return k;
}

void Registry::describe(const std::string& name, const std::string& help, const std::string& type) {
  std::lock_guard<std::mutex> g(mu_);
  meta_[name] = {help, type};
}

void Registry::inc(const std::string& name, const Labels& l, double v) {
  std::lock_guard<std::mutex> g(mu_);
  values_[name][key(l)] += v;
}

void Registry::set(const std::string& name, const Labels& l, double v) {
  std::lock_guard<std::mutex> g(mu_);
  values_[name][key(l)] = v;
}

void Registry::observe(const std::string& name, const Labels& l, double v) {
  std::lock_guard<std::mutex> g(mu_);
  Hist& h = hists_[name][key(l)];
  if (h.counts.empty()) h.counts.assign(kNBuckets, 0);
  for (int i = 0; i < kNBuckets; i++)
    if (v <= kBuckets[i]) h.counts[i] += 1;
  h.sum += v;
  h.n += 1;
}

double Registry::value(const std::string& name, const Labels& l) const {
  std::lock_guard<std::mutex> g(mu_);
  auto it = values_.find(name);
  if (it == values_.end()) return 0;
  auto jt = it->second.find(key(l));
  return jt == it->second.end() ? 0 : jt->second;
}

std::string Registry::exposition() const {
  std::lock_guard<std::mutex> g(mu_);
  std::string o;
  auto header = [&](const std::string& name, const char* dflt_type) {
    auto m = meta_.find(name);
    if (m != meta_.end()) {
      o += "# HELP " + name + " " + m->second.first + "\n# TYPE " + name + " " + m->second.second + "\n";
    } else {
      o += "# TYPE " + name + " " + dflt_type + "\n";
    }
  };
  for (auto& kv : values_) {
    header(kv.first, "gauge");
    for (auto& s : kv.second) {
      char num[64];
      snprintf(num, sizeof(num), "%.17g", s.second);
      o += kv.first + (s.first.empty() ? "" : "{" + s.first + "}") + " " + num + "\n";
    }
  }
  for (auto& kv : hists_) {
    header(kv.first, "histogram");
    for (auto& s : kv.second) {
      const std::string sep = s.first.empty() ? "" : ",";
      for (int i = 0; i < kNBuckets; i++) {
        char le[32];
        snprintf(le, sizeof(le), "%g", kBuckets[i]);
        o += kv.first + "_bucket{" + s.first + sep + "le=\"" + le + "\"} " + std::to_string((uint64_t)s.second.counts[i]) +
             "\n";
      }
      o += kv.first + "_bucket{" + s.first + sep + "le=\"+Inf\"} " + std::to_string(s.second.n) + "\n";
      char sum[64];
      snprintf(sum, sizeof(sum), "%.17g", s.second.sum);
      o += kv.first + "_sum" + (s.first.empty() ? "" : "{" + s.first + "}") + " " + sum + "\n";
      o += kv.first + "_count" + (s.first.empty() ? "" : "{" + s.first + "}") + " " + std::to_string(s.second.n) + "\n";
    }
  }
  return o;
}

static constexpr size_t kMaxBody = 16u << 20;  // a request body larger than this is refused

static bool read_request(tls::Stream& st, HttpRequest& req) {
  std::string buf;
  char tmp[8192];
  size_t header_end = std::string::npos;
  while (header_end == std::string::npos) {
    const long n = st.read_some(tmp, sizeof(tmp), 2000);
    if (n <= 0) return false;
    buf.append(tmp, size_t(n));
    header_end = buf.find("\r\n\r\n");
    if (buf.size() > (1 << 20)) return false;
  }
  const auto line_end = buf.find("\r\n");
  const std::string line = buf.substr(0, line_end);
  const auto sp1 = line.find(' '), sp2 = line.rfind(' ');
  if (sp1 == std::string::npos || sp2 == sp1) return false;
  req.method = line.substr(0, sp1);
  req.path = line.substr(sp1 + 1, sp2 - sp1 - 1);
  size_t content_len = 0;
  std::string headers = buf.substr(line_end + 2, header_end - line_end - 2);
  for (size_t p = 0; p < headers.size();) {
    size_t e = headers.find("\r\n", p);
    if (e == std::string::npos) e = headers.size();
    const std::string h = headers.substr(p, e - p);
    const auto colon = h.find(':');
    if (colon != std::string::npos) {
      std::string name = h.substr(0, colon), value = h.substr(colon + 1);
      for (auto& c : name) c = (char)tolower(c);
      while (!value.empty() && (value.front() == ' ' || value.front() == '\t')) value.erase(value.begin());
      if (name == "content-length") content_len = (size_t)atol(value.c_str());
      req.headers[name] = value;
    }
    p = e + 2;
  }
  if (content_len > kMaxBody) return false;
  req.body = buf.substr(header_end + 4);
  while (req.body.size() < content_len) {
    const long n = st.read_some(tmp, sizeof(tmp), 2000);
    if (n <= 0) return false;
    req.body.append(tmp, size_t(n));
  }
  return true;
}

static const char* reason(int s) {
  switch (s) {
    case 200: return "OK";
    case 201: return "Created";
    case 400: return "Bad Request";
    case 404: return "Not Found";
    case 409: return "Conflict";
    case 500: return "Internal Server Error";
    case 503: return "Service Unavailable";
    default: return "Error";
  }
}

// One connection: handshake, request, answer. /metrics and /healthz are answered here (the
// registry has its own lock); a route runs on the loop's thread, since it reads the process's
// state, and the connection waits for it at most 10 s.
static void serve_http_conn(Loop* loop, int fd, HttpRoute route, HttpOptions opt) {
  tls::Stream st;
  std::string terr;
  if (!tls::accept_stream(fd, 5000, st, &terr, opt.client_cert)) return;  // HTTPS when TLS is configured
  HttpRequest req;
  HttpResponse resp;
  if (!read_request(st, req)) {
    st.close();
    return;
  }
  const std::string path = req.path.substr(0, req.path.find('?'));
  if (opt.gate && !(path == "/healthz") && !opt.gate(req, resp)) {
    // refused: the gate set the answer
  } else if (req.method == "GET" && path == "/metrics") {
    resp.body = metrics().exposition();
  } else if (req.method == "GET" && path == "/healthz") {
    resp.body = "ok\n";
  } else if (route && !opt.route_on_loop) {
    if (!route(req, resp)) {
      resp.status = 404;
      resp.body = "not found\n";
    }
  } else if (route) {
    struct Pending {
      std::mutex mu;
      std::condition_variable cv;
      bool done = false, handled = false;
      HttpResponse resp;
    };
    auto pend = std::make_shared<Pending>();
    loop->post([pend, route, req] {
      HttpResponse r;
      const bool h = route(req, r);
      std::lock_guard<std::mutex> g(pend->mu);
      pend->resp = std::move(r);
      pend->handled = h;
      pend->done = true;
      pend->cv.notify_all();
    });
    std::unique_lock<std::mutex> lk(pend->mu);
    if (!pend->cv.wait_for(lk, std::chrono::seconds(10), [&] { return pend->done; })) {
      resp.status = 503;
      resp.body = "busy\n";
    } else if (pend->handled) {
      resp = pend->resp;
    } else {
      resp.status = 404;
      resp.body = "not found\n";
    }
  } else {
    resp.status = 404;
    resp.body = "not found\n";
  }
  std::string out = "HTTP/1.1 " + std::to_string(resp.status) + " " + reason(resp.status) +
                    "\r\nContent-Type: " + resp.content_type + "\r\nContent-Length: " + std::to_string(resp.body.size()) +
                    "\r\nConnection: close\r\n" + resp.extra_headers + "\r\n" + resp.body;
  st.write_all(out, 5000);
  st.close();
}

bool serve_http(Loop& loop, const std::string& addr, HttpRoute route, std::string* err, HttpOptions opt) {
  Address a;
  if (!Address::parse(addr, a)) {
    if (err) *err = "bad address " + addr;
    return false;
  }
  const int lfd = listen_on(a, err);
  if (lfd < 0) return false;
  // the listener blocks on its own thread; a slow client holds only its connection's thread,
  // never the loop (whose latency is the control plane's)
  const int flags = fcntl(lfd, F_GETFL, 0);
  fcntl(lfd, F_SETFL, flags & ~O_NONBLOCK);
  Loop* lp = &loop;
  std::thread([lfd, lp, route, opt] {
    static std::atomic<int> active{0};
    for (;;) {
      const int fd = ::accept4(lfd, nullptr, nullptr, SOCK_CLOEXEC);
      if (fd < 0) {
        if (errno == EINTR || errno == ECONNABORTED || errno == EMFILE || errno == ENFILE) {
          if (errno == EMFILE || errno == ENFILE) usleep(10000);
          continue;
        }
        return;
      }
      if (active.load() >= 64) {  // bounded: beyond this, connections wait their turn here
        serve_http_conn(lp, fd, route, opt);
        continue;
      }
      active++;
      std::thread([lp, fd, route, opt] {
        serve_http_conn(lp, fd, route, opt);
        active--;
      }).detach();
    }
  }).detach();
  return true;
}

static std::string dechunk(const std::string& b) {
  std::string out;
  size_t i = 0;
  while (i < b.size()) {
    const size_t le = b.find("\r\n", i);
    if (le == std::string::npos) break;
    const size_t n = std::strtoul(b.substr(i, le - i).c_str(), nullptr, 16);
    if (n == 0) break;
    out += b.substr(le + 2, n);
    i = le + 2 + n + 2;
  }
  return out;
}

// One request over a connected stream; the answer's status (-1: none) and body.
static int exchange(tls::Stream& st, const std::string& host, const std::string& method, const std::string& path,
                    const std::vector<std::string>& headers, const std::string& body, std::string& out,
                    int timeout_ms) {
  std::string req = method + " " + path + " HTTP/1.1\r\nHost: " + host + "\r\nContent-Length: " +
                    std::to_string(body.size()) + "\r\nConnection: close\r\n";
  for (auto& h : headers) req += h + "\r\n";
  req += "\r\n" + body;
  const uint64_t deadline = now_ms() + (uint64_t)timeout_ms;
  if (!st.write_all(req, timeout_ms)) {
    st.close();
    return -1;
  }
  std::string resp;
  char tmp[8192];
  while (now_ms() < deadline) {
    const long n = st.read_some(tmp, sizeof(tmp), (int)std::max<int64_t>(1, (int64_t)(deadline - now_ms())));
    if (n <= 0) break;
    resp.append(tmp, size_t(n));
  }
  st.close();
  const auto sp = resp.find(' ');
  if (sp == std::string::npos) return -1;
  const int status = atoi(resp.c_str() + sp + 1);
  const auto be = resp.find("\r\n\r\n");
  if (be == std::string::npos) {
    out.clear();
    return status;
  }
  std::string head = resp.substr(0, be);
  for (auto& c : head) c = (char)std::tolower((unsigned char)c);
  out = resp.substr(be + 4);
  if (head.find("transfer-encoding: chunked") != std::string::npos) out = dechunk(out);
  return status;
}

int http_request_ex(const std::string& addr, const std::string& method, const std::string& path,
                    const std::vector<std::string>& headers, const std::string& body, std::string& out, int timeout_ms) {
  Address a;
  if (!Address::parse(addr, a)) return -1;
  tls::Stream st;
  if (!tls::connect_stream(a, timeout_ms, st, nullptr)) return -1;
  return exchange(st, a.host, method, path, headers, body, out, timeout_ms);
}

bool parse_url(const std::string& url, bool& https, std::string& hostport, std::string& path) {
  std::string rest = url;
  https = false;
  if (rest.rfind("https://", 0) == 0) {
    https = true;
    rest = rest.substr(8);
  } else if (rest.rfind("http://", 0) == 0) {
    rest = rest.substr(7);
  }
  const auto slash = rest.find('/');
  hostport = rest.substr(0, slash);
  path = slash == std::string::npos ? "/" : rest.substr(slash);
  if (hostport.empty()) return false;
  if (hostport.find(':') == std::string::npos) hostport += https ? ":443" : ":80";
  return true;
}

int http_url(const std::string& url, const std::string& method, const std::vector<std::string>& headers,
             const std::string& body, std::string& out, int timeout_ms, const std::string& ca_file) {
  bool https = false;
  std::string hostport, path;
  Address a;
  if (!parse_url(url, https, hostport, path) || !Address::parse(hostport, a)) return -1;
  tls::Stream st;
  if (!tls::connect_web(a, https, ca_file, timeout_ms, st, nullptr)) return -1;
  return exchange(st, a.host, method, path, headers, body, out, timeout_ms);
}

int http_request(const std::string& addr, const std::string& method, const std::string& path, const std::string& body,
                 std::string& out) {
  return http_request_ex(addr, method, path, {}, body, out, 8000);
}

}  // namespace es
