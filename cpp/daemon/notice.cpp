#include "notice.h"

#include <time.h>

#include <chrono>
#include <vector>

#include "kube.h"
#include "net.h"
#include "telemetry.h"
#include "util.h"

namespace es {

static int64_t wall_ms() {
  return std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::system_clock::now().time_since_epoch())
      .count();
}

int64_t parse_time_ms(const std::string& s) {
  struct tm tm = {};
  const char* end = strptime(s.c_str(), "%Y-%m-%dT%H:%M:%S", &tm);
  if (end == nullptr) end = strptime(s.c_str(), "%a, %d %b %Y %H:%M:%S", &tm);
  if (end == nullptr) return 0;
  return (int64_t)timegm(&tm) * 1000;
}

NoticeWatcher::NoticeWatcher(std::string source, std::string endpoint, std::string node, uint32_t interval_ms)
    : source_(std::move(source)), endpoint_(std::move(endpoint)), node_(std::move(node)), interval_ms_(interval_ms) {
  if (endpoint_.empty()) {
    if (source_ == "aws" || source_ == "azure") endpoint_ = "http://169.254.169.254";
    else if (source_ == "gcp") endpoint_ = "http://metadata.google.internal";
  } else if (endpoint_.find("://") == std::string::npos) {
    endpoint_ = "http://" + endpoint_;
  }
}

// A metadata endpoint is plain HTTP on the link-local network, never the cluster's mutual TLS.
int NoticeWatcher::get(const std::string& method, const std::string& path, const std::vector<std::string>& headers,
                       std::string& body) {
  if (source_ == "k8s") {
    const KubeClient k = endpoint_.empty() ? KubeClient::from_env() : KubeClient::at(endpoint_);
    return k.request(method, path, "", body);
  }
  return http_url(endpoint_ + path, method, headers, "", body);
}

NoticeWatcher::~NoticeWatcher() {
  stop_ = true;
  if (thread_.joinable()) thread_.join();
}

bool NoticeWatcher::start(std::string* err) {
  if (source_ != "aws" && source_ != "gcp" && source_ != "azure" && source_ != "k8s") {
    if (err) *err = "unknown notice source " + source_ + " (aws, gcp, azure, k8s)";
    return false;
  }
  thread_ = std::thread([this] { run(); });
  return true;
}

bool NoticeWatcher::take(NodeNoticeEvent& out) {
  std::lock_guard<std::mutex> g(mu_);
  if (!pending_) return false;
  pending_ = false;
  out = event_;
  return true;
}

void NoticeWatcher::run() {
  while (!stop_) {
    NodeNoticeEvent ev;
    if (poll_once(ev)) {
      std::lock_guard<std::mutex> g(mu_);
      if (!reported_) {  // one notice per departure: the node is draining from then on
        event_ = ev;
        pending_ = reported_ = true;
      }
    }
    for (uint32_t t = 0; t < interval_ms_ && !stop_; t += 50) std::this_thread::sleep_for(std::chrono::milliseconds(50));
  }
}

bool NoticeWatcher::poll_once(NodeNoticeEvent& out) {
  std::string body;
  out.source = source_;
  if (source_ == "aws") {
    std::string token;
    if (get("PUT", "/latest/api/token", {"X-aws-ec2-metadata-token-ttl-seconds: 300"}, token) != 200)
      return false;
    const int st = get("GET", "/latest/meta-data/spot/instance-action", {"X-aws-ec2-metadata-token: " + token}, body);
    if (st != 200) return false;
    Json j;
    if (!Json::parse(body, j)) return false;
    const Json* action = j.get("action");
    const Json* t = j.get("time");
    out.detail = "spot " + (action ? action->str : std::string("action"));
    out.deadline_ms = t ? parse_time_ms(t->str) : 0;
    if (out.deadline_ms == 0) out.deadline_ms = wall_ms() + 120000;
    return true;
  }
  if (source_ == "gcp") {
    const std::vector<std::string> h = {"Metadata-Flavor: Google"};
    if (get("GET", "/computeMetadata/v1/instance/preempted", h, body) == 200 &&
        body.find("TRUE") != std::string::npos) {
      out.detail = "preempted";
      out.deadline_ms = wall_ms() + 30000;
      return true;
    }
    if (get("GET", "/computeMetadata/v1/instance/maintenance-event", h, body) == 200 &&
        !body.empty() && body.find("NONE") == std::string::npos) {
      out.detail = "maintenance " + body.substr(0, 64);
      out.deadline_ms = wall_ms() + 60000;
      return true;
    }
    return false;
  }
  if (source_ == "azure") {
    if (get("GET", "/metadata/scheduledevents?api-version=2020-07-01", {"Metadata: true"}, body) != 200)
      return false;
    Json j;
    if (!Json::parse(body, j)) return false;
    const Json* evs = j.get("Events");
    if (!evs) return false;
    for (auto& e : evs->arr) {
      const Json* type = e.get("EventType");
      if (!type) continue;
      const std::string& t = type->str;
      if (t != "Preempt" && t != "Terminate" && t != "Reboot" && t != "Redeploy") continue;
      const Json* nb = e.get("NotBefore");
      out.detail = t;
      out.deadline_ms = nb && !nb->str.empty() ? parse_time_ms(nb->str) : 0;
      if (out.deadline_ms == 0) out.deadline_ms = wall_ms() + 30000;
      return true;
    }
    return false;
  }
  // k8s: the node object
  if (get("GET", "/api/v1/nodes/" + node_, {}, body) != 200)
    return false;
  Json j;
  if (!Json::parse(body, j)) return false;
  const Json* spec = j.get("spec");
  if (!spec) return false;
  if (const Json* u = spec->get("unschedulable"); u && u->b) {
    out.detail = "cordoned";
    out.deadline_ms = wall_ms() + 30000;
    return true;
  }
  if (const Json* taints = spec->get("taints")) {
    for (auto& t : taints->arr) {
      const Json* k = t.get("key");
      if (!k) continue;
      const std::string& key = k->str;
      if (key == "ToBeDeletedByClusterAutoscaler" || key == "node.kubernetes.io/unschedulable" ||
          key == "cloud.google.com/impending-node-termination" || key == "aws-node-termination-handler/spot-itn" ||
          key == "karpenter.sh/disruption") {
        out.detail = "taint " + key;
        out.deadline_ms = wall_ms() + 30000;
        return true;
      }
    }
  }
  return false;
}

}  // namespace es
