// Who may use the operator API when it is not gated by client certificates (--api-auth kube):
// a bearer token, reviewed by the Kubernetes API server (TokenReview: who is it), then
// authorized by it (SubjectAccessReview: may that user do this verb on this resource of group
// everserve.ai in the namespace). GET, and the watch feed, are `get`/`list`/`watch`; PUT is
// `update`, POST `create`, DELETE `delete`; the resource is the path's (engines, nodes, pools,
// stacks). Answers are kept for 30 s per (token digest, verb, resource) so a busy operator does
// not load the API server; a caller beyond 16 reviews in flight is told to come back (503).
//
// Reference parity: controller/src/api/kubernetes.rs (TokenReview identity, access review,
// cache keyed by the token's digest, bounded reviews).
#pragma once

#include <atomic>
#include <map>
#include <mutex>
#include <string>

#include "kube.h"
#include "telemetry.h"

namespace es {

class KubeGate {
 public:
  KubeGate(KubeClient k, std::string ns) : k_(std::move(k)), ns_(std::move(ns)) {}
  bool admit(const HttpRequest& req, HttpResponse& resp);  // thread-safe

 private:
  struct Verdict {
    bool allowed = false;
    std::string why;
    uint64_t until_ms = 0;
  };
  bool review(const std::string& token, const std::string& verb, const std::string& resource, std::string& why);
  KubeClient k_;
  std::string ns_;
  std::mutex mu_;
  std::map<std::string, Verdict> cache_;
  std::atomic<int> in_flight_{0};
};

// (verb, resource) of an operator API request.
std::pair<std::string, std::string> access_of(const std::string& method, const std::string& path);

}  // namespace es
