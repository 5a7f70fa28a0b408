// Node enrollment on Kubernetes: a node daemon is issued its certificate by the coordinator.
//
//   POST /v1/certificates/node   Authorization: Bearer <the pod's projected service-account
//                                token, audience "everserve">   body {"publicKey": "<PEM>"}
//   200 {"node", "certificate", "ca", "notAfterMs"}
//
// The coordinator asks the API server's TokenReview who the token is, and signs, with the
// deployment's CA, a certificate for the node the API server says the token's pod runs on
// (`authentication.kubernetes.io/node-name`). Nothing the caller says chooses the name: a token
// from a pod on node-a gets node-a's certificate or none; a token the API server does not
// authenticate, for another audience, or not bound to a pod on a node is refused (401). The
// endpoint asks for no client certificate (the node has none yet), so it bounds what any caller
// can make it do: bodies of at most 4096 bytes, a bearer that is not shaped as a JWT refused
// unread, and at most 16 reviews in flight (503 with Retry-After beyond them).
//
// Reference parity: controller/src/issuer.rs and controller/src/enroll.rs (the same flow: key
// made and kept on the node, public half and token sent, certificate for the reviewed node).
#pragma once

#include <atomic>
#include <string>

#include "kube.h"
#include "telemetry.h"

namespace es {

constexpr const char* kEnrollPath = "/v1/certificates/node";
constexpr const char* kEnrollAudience = "everserve";

class Issuer {
 public:
  Issuer(KubeClient k, std::string ca_dir, int hours) : k_(std::move(k)), ca_dir_(std::move(ca_dir)), hours_(hours) {}
  // The route (thread-safe; it blocks on the API server, so it runs off the loop).
  bool route(const HttpRequest& req, HttpResponse& resp);

 private:
  KubeClient k_;
  std::string ca_dir_;
  int hours_;
  std::atomic<int> in_flight_{0};
};

// Whether `t` is shaped as a JWT (three base64url parts, at most 16 KiB).
bool jwt_shaped(const std::string& t);

}  // namespace es
