#include "api_auth.h"

#include <algorithm>

#include "issuer.h"
#include "net.h"
#include "tls.h"
#include "util.h"

namespace es {

std::pair<std::string, std::string> access_of(const std::string& method, const std::string& path) {
  std::string p = path.substr(0, path.find('?'));
  std::string resource = "engines";
  if (p.rfind("/v1/", 0) == 0) {
    const std::string rest = p.substr(4);
    resource = rest.substr(0, rest.find('/'));
    if (resource == "watch" || resource == "openapi") resource = "engines";
    if (rest.find("/stacks") != std::string::npos || resource == "stacks") resource = "stacks";
  }
  std::string verb = "get";
  if (method == "PUT") verb = "update";
  else if (method == "POST") verb = "create";
  else if (method == "DELETE") verb = "delete";
  else if (p == "/v1/watch") verb = "watch";
  else if (p.size() > 4 && std::count(p.begin(), p.end(), '/') == 2) verb = "list";
  return {verb, resource};
}

bool KubeGate::review(const std::string& token, const std::string& verb, const std::string& resource,
                      std::string& why) {
  std::string out;
  const std::string tr = "{\"apiVersion\":\"authentication.k8s.io/v1\",\"kind\":\"TokenReview\",\"spec\":{\"token\":\"" +
                         json_escape(token) + "\"}}";
  const int st = k_.request("POST", "/apis/authentication.k8s.io/v1/tokenreviews", tr, out);
  Json r;
  if ((st != 200 && st != 201) || !Json::parse(out, r)) {
    why = "the API server did not review the token (" + std::to_string(st) + ")";
    return false;
  }
  const Json* status = r.get("status");
  const Json* ok = status ? status->get("authenticated") : nullptr;
  const Json* user = status ? status->get("user") : nullptr;
  const Json* name = user ? user->get("username") : nullptr;
  if (!ok || !ok->b || !name || name->str.empty()) {
    why = "the token is not authenticated";
    return false;
  }
  std::string groups = "[";
  if (const Json* gs = user->get("groups"))
    for (size_t i = 0; i < gs->arr.size(); i++) groups += (i ? ",\"" : "\"") + json_escape(gs->arr[i].str) + "\"";
  groups += "]";
  const std::string sar =
      "{\"apiVersion\":\"authorization.k8s.io/v1\",\"kind\":\"SubjectAccessReview\",\"spec\":{\"user\":\"" +
      json_escape(name->str) + "\",\"groups\":" + groups + ",\"resourceAttributes\":{\"namespace\":\"" +
      json_escape(ns_) + "\",\"group\":\"everserve.ai\",\"resource\":\"" + json_escape(resource) + "\",\"verb\":\"" +
      json_escape(verb) + "\"}}}";
  const int as = k_.request("POST", "/apis/authorization.k8s.io/v1/subjectaccessreviews", sar, out);
  Json a;
  if ((as != 200 && as != 201) || !Json::parse(out, a)) {
    why = "the API server did not review the access (" + std::to_string(as) + ")";
    return false;
  }
  const Json* ast = a.get("status");
  const Json* allowed = ast ? ast->get("allowed") : nullptr;
  if (!allowed || !allowed->b) {
    why = name->str + " may not " + verb + " " + resource;
    return false;
  }
  return true;
}

bool KubeGate::admit(const HttpRequest& req, HttpResponse& resp) {
  auto refuse = [&](int code, const std::string& why) {
    resp.status = code;
    resp.content_type = "application/json";
    resp.body = "{\"error\":\"" + json_escape(why) + "\"}";
    metrics().inc("everserve_api_refusals_total", {{"code", std::to_string(code)}});
    return false;
  };
  auto auth = req.headers.find("authorization");
  if (auth == req.headers.end() || auth->second.rfind("Bearer ", 0) != 0) return refuse(401, "a bearer token is needed");
  const std::string token = auth->second.substr(7);
  if (!jwt_shaped(token)) return refuse(401, "the bearer is not a token");
  const auto [verb, resource] = access_of(req.method, req.path);
  const std::string key = sha256_hex(token) + "|" + verb + "|" + resource;
  const uint64_t now = now_ms();
  {
    std::lock_guard<std::mutex> g(mu_);
    auto it = cache_.find(key);
    if (it != cache_.end() && it->second.until_ms > now)
      return it->second.allowed ? true : refuse(403, it->second.why);
    if (cache_.size() > 4096) cache_.clear();
  }
  if (in_flight_.fetch_add(1) >= 16) {
    in_flight_.fetch_sub(1);
    resp.extra_headers = "Retry-After: 1\r\n";
    return refuse(503, "too many reviews in flight");
  }
  std::string why;
  const bool ok = review(token, verb, resource, why);
  in_flight_.fetch_sub(1);
  {
    std::lock_guard<std::mutex> g(mu_);
    cache_[key] = {ok, why, now + 30000};
  }
  return ok ? true : refuse(why.rfind("the token", 0) == 0 || why.rfind("the API", 0) == 0 ? 401 : 403, why);
}

}  // namespace es
