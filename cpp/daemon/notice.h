// Notices of a node's coming departure, from the cloud or cluster it runs in.
//
// A watcher polls one source on its own thread (the daemon's loop never blocks on HTTP) and
// hands the loop each new notice once. Sources, with the endpoints they read (an
// `--notice-endpoint URL` or `host:port` replaces the well-known address, e.g. for a local fake;
// metadata services are plain HTTP, never the cluster's mutual TLS):
//   aws    IMDSv2: a session token (PUT /latest/api/token), then
//          GET /latest/meta-data/spot/instance-action -> {"action": ..., "time": ISO-8601}
//   gcp    GET /computeMetadata/v1/instance/preempted ("TRUE") and .../maintenance-event
//          (anything but "NONE"); header Metadata-Flavor: Google; 30 s of notice
//   azure  GET /metadata/scheduledevents?api-version=2020-07-01 (header Metadata: true):
//          events of type Preempt, Terminate, Reboot or Redeploy; NotBefore is the deadline
//   k8s    GET /api/v1/nodes/<node> from the Kubernetes API (kube.h: in-cluster service account,
//          EVERSERVE_KUBE_API, or kubectl proxy): the node unschedulable, or tainted for deletion /
//          termination
#pragma once

#include <atomic>
#include <cstdint>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace es {

struct NodeNoticeEvent {
  std::string source;
  int64_t deadline_ms = 0;  // wall-clock ms
  std::string detail;
};

class NoticeWatcher {
 public:
  NoticeWatcher(std::string source, std::string endpoint, std::string node, uint32_t interval_ms);
  ~NoticeWatcher();
  bool start(std::string* err);
  // A notice not handed out yet (called from the daemon's loop).
  bool take(NodeNoticeEvent& out);

  // One poll of the source (exposed for tests); true and `out` filled when a notice is current.
  bool poll_once(NodeNoticeEvent& out);

 private:
  int get(const std::string& method, const std::string& path, const std::vector<std::string>& headers,
          std::string& body);
  void run();
  std::string source_, endpoint_, node_;
  uint32_t interval_ms_;
  std::thread thread_;
  std::atomic<bool> stop_{false};
  std::mutex mu_;
  bool pending_ = false, reported_ = false;
  NodeNoticeEvent event_;
};

// "2026-12-01T22:00:00Z" or an RFC 1123 date ("Mon, 01 Dec 2026 22:00:00 GMT") to ms since the
// epoch; 0 when it parses as neither.
int64_t parse_time_ms(const std::string& s);

}  // namespace es
