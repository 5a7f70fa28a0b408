#include "issuer.h"

#include "tls.h"
#include "util.h"

namespace es {

bool jwt_shaped(const std::string& t) {
  if (t.empty() || t.size() > 16384) return false;
  int dots = 0;
  for (char c : t) {
    if (c == '.') dots++;
    else if (!(isalnum((unsigned char)c) || c == '-' || c == '_' || c == '=')) return false;
  }
  return dots == 2;
}

static void answer(HttpResponse& resp, int status, const std::string& why) {
  resp.status = status;
  resp.content_type = "application/json";
  resp.body = "{\"error\":\"" + json_escape(why) + "\"}";
}

bool Issuer::route(const HttpRequest& req, HttpResponse& resp) {
  if (req.path.substr(0, req.path.find('?')) != kEnrollPath) return false;
  if (req.method != "POST") {
    answer(resp, 400, "POST a public key");
    return true;
  }
  if (req.body.size() > 4096) {
    answer(resp, 400, "the body is larger than 4096 bytes");
    return true;
  }
  auto auth = req.headers.find("authorization");
  std::string token = auth == req.headers.end() ? "" : auth->second;
  if (token.rfind("Bearer ", 0) != 0 || !jwt_shaped(token = token.substr(7))) {
    answer(resp, 401, "a bearer service-account token is needed");
    metrics().inc("everserve_enrollments_total", {{"verdict", "refused"}});
    return true;
  }
  Json body;
  std::string err;
  const Json* pk = nullptr;
  if (!Json::parse(req.body, body, &err) || !(pk = body.get("publicKey")) || pk->str.empty()) {
    answer(resp, 400, "the body is {\"publicKey\": PEM}");
    return true;
  }
  if (in_flight_.fetch_add(1) >= 16) {
    in_flight_.fetch_sub(1);
    answer(resp, 503, "too many reviews in flight");
    resp.extra_headers = "Retry-After: 1\r\n";
    return true;
  }
  struct Release {
    std::atomic<int>& n;
    ~Release() { n.fetch_sub(1); }
  } release{in_flight_};
  const std::string review = "{\"apiVersion\":\"authentication.k8s.io/v1\",\"kind\":\"TokenReview\",\"spec\":{\"token\":\"" +
                             json_escape(token) + "\",\"audiences\":[\"" + kEnrollAudience + "\"]}}";
  std::string out;
  const int st = k_.request("POST", "/apis/authentication.k8s.io/v1/tokenreviews", review, out);
  Json r;
  if ((st != 200 && st != 201) || !Json::parse(out, r)) {
    answer(resp, 503, "the API server did not review the token (" + std::to_string(st) + ")");
    resp.extra_headers = "Retry-After: 2\r\n";
    return true;
  }
  const Json* status = r.get("status");
  const Json* ok = status ? status->get("authenticated") : nullptr;
  const Json* user = status ? status->get("user") : nullptr;
  const Json* extra = user ? user->get("extra") : nullptr;
  const Json* node = extra ? extra->get("authentication.kubernetes.io/node-name") : nullptr;
  bool audience = false;
  if (const Json* auds = status ? status->get("audiences") : nullptr)
    for (auto& a : auds->arr) audience |= a.str == kEnrollAudience;
  if (!ok || !ok->b || !audience || !node || node->arr.empty() || node->arr[0].str.empty()) {
    answer(resp, 401, "the token is not a pod's on a node, for audience everserve");
    metrics().inc("everserve_enrollments_total", {{"verdict", "refused"}});
    return true;
  }
  const std::string name = node->arr[0].str;
  std::string cert, ca;
  int64_t not_after = 0;
  if (!tls::sign_node(ca_dir_, name, pk->str, hours_, cert, ca, not_after, &err)) {
    answer(resp, 400, err);
    return true;
  }
  resp.content_type = "application/json";
  resp.body = "{\"node\":\"" + json_escape(name) + "\",\"certificate\":\"" + json_escape(cert) + "\",\"ca\":\"" +
              json_escape(ca) + "\",\"notAfterMs\":" + std::to_string(not_after) + "}";
  metrics().inc("everserve_enrollments_total", {{"verdict", "issued"}});
  ES_INFO("issued node %s its certificate (valid %d h)", name.c_str(), hours_);
  return true;
}

}  // namespace es
