// Per-process telemetry: a Prometheus registry (counters, gauges, histograms with labels) and a
// small HTTP endpoint serving /metrics, /healthz and any routes a process adds (the coordinator's
// operator API). Metric names are stable: add, never rename.
#pragma once

#include <cstdint>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <vector>

namespace es {

using Labels = std::vector<std::pair<std::string, std::string>>;

class Registry {
 public:
  void describe(const std::string& name, const std::string& help, const std::string& type);
  void inc(const std::string& name, const Labels& l = {}, double v = 1.0);
  void set(const std::string& name, const Labels& l, double v);
  void observe(const std::string& name, const Labels& l, double v);  // histogram (seconds buckets)
  double value(const std::string& name, const Labels& l = {}) const;
  std::string exposition() const;

 private:
  struct Hist {
    std::vector<double> counts;
    double sum = 0;
    uint64_t n = 0;
  };
  static std::string key(const Labels& l);
  mutable std::mutex mu_;
  std::map<std::string, std::pair<std::string, std::string>> meta_;  // name -> help, type
  std::map<std::string, std::map<std::string, double>> values_;
  std::map<std::string, std::map<std::string, Hist>> hists_;
};

Registry& metrics();

struct HttpRequest {
  std::string method, path, body;
  std::map<std::string, std::string> headers;  // names in lower case
};
struct HttpResponse {
  int status = 200;
  std::string content_type = "text/plain; version=0.0.4";
  std::string body;
  std::string extra_headers;  // "Name: value\r\n" lines
};
struct HttpOptions {
  bool client_cert = true;    // ask for a client certificate when TLS is configured
  bool route_on_loop = true;  // the route reads the loop's state: run it there (else on the
                              // connection's thread, for routes that block, e.g. on another API)
  // Runs on the connection's thread before the route (it may block, e.g. on a token review):
  // false refuses the request with the status and body it set.
  std::function<bool(const HttpRequest&, HttpResponse&)> gate;
};
using HttpRoute = std::function<bool(const HttpRequest&, HttpResponse&)>;  // true: handled

class Loop;
// Serve HTTP on `addr` ("host:port") from `loop`: /metrics, /healthz, then `route`.
bool serve_http(Loop& loop, const std::string& addr, HttpRoute route = nullptr, std::string* err = nullptr,
                HttpOptions opt = {});
// A blocking HTTP request (used by the CLI); returns the status code, or -1.
int http_request(const std::string& addr, const std::string& method, const std::string& path, const std::string& body,
                 std::string& out);
// The same with extra request headers ("Name: value" lines) and a bound on the whole exchange;
// chunked response bodies are decoded.
int http_request_ex(const std::string& addr, const std::string& method, const std::string& path,
                    const std::vector<std::string>& headers, const std::string& body, std::string& out,
                    int timeout_ms = 2000);

// A request to a web endpoint outside the control plane (cloud metadata, the Kubernetes API):
// `url` is http://host[:port]/path (plain) or https://... (server verified against `ca_file`,
// the system's trust store when empty); never the cluster's mutual TLS.
int http_url(const std::string& url, const std::string& method, const std::vector<std::string>& headers,
             const std::string& body, std::string& out, int timeout_ms = 5000, const std::string& ca_file = "");
// "http(s)://host[:port]/path" into its parts (the default port of the scheme when none).
bool parse_url(const std::string& url, bool& https, std::string& hostport, std::string& path);

}  // namespace es
