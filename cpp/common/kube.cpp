#include "kube.h"

#include <time.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>

#include "telemetry.h"
#include "util.h"

namespace es {

static const char* kServiceAccount = "/var/run/secrets/kubernetes.io/serviceaccount";

KubeClient KubeClient::from_env() {
  KubeClient k;
  const std::string api = env_or("EVERSERVE_KUBE_API", "");
  if (!api.empty()) {
    k.base = api;
    k.token_file = env_or("EVERSERVE_KUBE_TOKEN_FILE", "");
    k.ca = env_or("EVERSERVE_KUBE_CA", "");
    return k;
  }
  const std::string host = env_or("KUBERNETES_SERVICE_HOST", "");
  if (!host.empty()) {
    const std::string port = env_or("KUBERNETES_SERVICE_PORT", "443");
    k.base = "https://" + (host.find(':') != std::string::npos ? "[" + host + "]" : host) + ":" + port;
    k.token_file = std::string(kServiceAccount) + "/token";
    k.ca = std::string(kServiceAccount) + "/ca.crt";
    return k;
  }
  k.base = "http://127.0.0.1:8001";
  return k;
}

KubeClient KubeClient::at(const std::string& url) {
  KubeClient k;
  k.base = url.find("://") == std::string::npos ? "http://" + url : url;
  return k;
}

int KubeClient::request(const std::string& method, const std::string& path, const std::string& body,
                        std::string& out, int timeout_ms) const {
  std::vector<std::string> headers = {"Accept: application/json"};
  if (!body.empty()) headers.push_back(method == "PATCH" ? "Content-Type: application/merge-patch+json"
                                                          : "Content-Type: application/json");
  if (!token_file.empty()) {
    std::string tok;
    if (read_file(token_file, tok)) {
      while (!tok.empty() && (tok.back() == '\n' || tok.back() == '\r' || tok.back() == ' ')) tok.pop_back();
      headers.push_back("Authorization: Bearer " + tok);
    }
  }
  return http_url(base + path, method, headers, body, out, timeout_ms, ca);
}

int64_t wall_clock_ms() {
  return std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::system_clock::now().time_since_epoch())
      .count();
}

std::string rfc3339_micro(int64_t wall_ms) {
  const time_t secs = (time_t)(wall_ms / 1000);
  struct tm tm;
  gmtime_r(&secs, &tm);
  char buf[64];
  std::snprintf(buf, sizeof buf, "%04d-%02d-%02dT%02d:%02d:%02d.%06dZ", tm.tm_year + 1900, tm.tm_mon + 1, tm.tm_mday,
                tm.tm_hour, tm.tm_min, tm.tm_sec, (int)(wall_ms % 1000) * 1000);
  return buf;
}

int64_t parse_rfc3339_ms(const std::string& s) {
  struct tm tm = {};
  const char* end = strptime(s.c_str(), "%Y-%m-%dT%H:%M:%S", &tm);
  if (end == nullptr) return 0;
  int64_t ms = (int64_t)timegm(&tm) * 1000;
  if (*end == '.') {
    int digits = 0, frac = 0;
    for (const char* p = end + 1; *p >= '0' && *p <= '9'; p++)
      if (digits < 3) {
        frac = frac * 10 + (*p - '0');
        digits++;
      }
    while (digits < 3) {
      frac *= 10;
      digits++;
    }
    ms += frac;
  }
  return ms;
}

}  // namespace es
