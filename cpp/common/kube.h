// A small client of the Kubernetes API (JSON over HTTP/1.1) for what the control plane asks of
// it: node objects (notices), Lease objects (the coordinator's lease) and TokenReviews (node
// enrollment).
//
// Where it connects: EVERSERVE_KUBE_API (a URL; with EVERSERVE_KUBE_TOKEN_FILE and
// EVERSERVE_KUBE_CA), else the in-cluster service (KUBERNETES_SERVICE_HOST / _PORT, the pod's
// service-account token and CA under /var/run/secrets/kubernetes.io/serviceaccount), else a
// local `kubectl proxy` at http://127.0.0.1:8001. The token is read again for every request
// (projected tokens rotate).
#pragma once

#include <string>

namespace es {

struct KubeClient {
  std::string base;        // "https://host:port" or "http://host:port"
  std::string token_file;  // bearer token ("" none)
  std::string ca;          // CA of the API server (https)
  static KubeClient from_env();
  static KubeClient at(const std::string& url);  // a given endpoint, no token
  // The answer's status (-1: no answer) and body.
  int request(const std::string& method, const std::string& path, const std::string& body, std::string& out,
              int timeout_ms = 5000) const;
};

// "2026-12-02T10:00:00.123456Z" (RFC 3339, as MicroTime) for wall-clock ms.
std::string rfc3339_micro(int64_t wall_ms);
// RFC 3339 ("...T10:00:00Z", fractions of a second kept to the millisecond) to wall-clock ms;
// 0 when it does not parse.
int64_t parse_rfc3339_ms(const std::string& s);
int64_t wall_clock_ms();

}  // namespace es
