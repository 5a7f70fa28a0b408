#include "lease.h"

#include <fcntl.h>
#include <sys/file.h>
#include <unistd.h>

#include <chrono>
#include <cstdlib>
#include <thread>

#include "everserve_pb.h"
#include "net.h"
#include "telemetry.h"
#include "util.h"

namespace es {

namespace {

class FileLease : public Lease {
 public:
  FileLease(std::string path, std::string holder) : path_(std::move(path)), holder_(std::move(holder)) {}
  bool acquire(uint64_t& term, std::string& err) override {
    const int fd = ::open(path_.c_str(), O_RDWR | O_CREAT | O_CLOEXEC, 0660);
    if (fd < 0) {
      err = "cannot open the lease " + path_;
      return false;
    }
    while (flock(fd, LOCK_EX | LOCK_NB) != 0) {
      ES_INFO("waiting for the lease %s", path_.c_str());
      sleep(1);
    }
    std::string data;
    char buf[4096];
    ssize_t n;
    while ((n = ::read(fd, buf, sizeof(buf))) > 0) data.append(buf, size_t(n));
    coord::LeaseRecord rec;
    if (!data.empty()) rec.parse(data);
    rec.term += 1;
    rec.holder = holder_;
    rec.renewed_at_ms = (int64_t)now_ms();
    const std::string out = rec.serialize();
    if (ftruncate(fd, 0) != 0 || pwrite(fd, out.data(), out.size(), 0) != (ssize_t)out.size()) {
      err = "cannot write the lease";
      return false;
    }
    fsync(fd);
    term = rec.term;
    return true;  // the fd stays open (and locked) until exit
  }

 private:
  std::string path_, holder_;
};

}  // namespace

std::unique_ptr<Lease> make_lease(const std::string& spec, const std::string& holder, uint32_t duration_s) {
  if (spec.rfind("etcd:", 0) == 0) {
    // etcd:http://host:2379/path/of/key
    const std::string rest = spec.substr(5);
    const auto scheme = rest.find("://");
    const auto slash = rest.find('/', scheme == std::string::npos ? 0 : scheme + 3);
    const std::string url = slash == std::string::npos ? rest : rest.substr(0, slash);
    const std::string key = slash == std::string::npos ? "/everserve/coordinator" : rest.substr(slash);
    return std::make_unique<EtcdLease>(url, key, holder, duration_s);
  }
  if (spec.rfind("k8s:", 0) == 0) {
    const std::string rest = spec.substr(4);
    const auto slash = rest.find('/');
    const std::string ns = slash == std::string::npos ? "default" : rest.substr(0, slash);
    const std::string name = slash == std::string::npos ? rest : rest.substr(slash + 1);
    return std::make_unique<KubeLease>(KubeClient::from_env(), ns, name, holder, duration_s);
  }
  return std::make_unique<FileLease>(spec, holder);
}

KubeLease::KubeLease(KubeClient k, std::string ns, std::string name, std::string holder, uint32_t duration_s)
    : k_(std::move(k)), ns_(std::move(ns)), name_(std::move(name)), holder_(std::move(holder)),
      duration_s_(duration_s ? duration_s : 15) {}

std::string KubeLease::path() const {
  return "/apis/coordination.k8s.io/v1/namespaces/" + ns_ + "/leases";
}

std::string KubeLease::body(uint64_t transitions, int64_t acquired_ms, int64_t renewed_ms) const {
  std::string meta = "{\"name\":\"" + json_escape(name_) + "\",\"namespace\":\"" + json_escape(ns_) + "\"";
  if (!rv_.empty()) meta += ",\"resourceVersion\":\"" + json_escape(rv_) + "\"";
  meta += "}";
  return "{\"apiVersion\":\"coordination.k8s.io/v1\",\"kind\":\"Lease\",\"metadata\":" + meta +
         ",\"spec\":{\"holderIdentity\":\"" + json_escape(holder_) + "\",\"leaseDurationSeconds\":" +
         std::to_string(duration_s_) + ",\"acquireTime\":\"" + rfc3339_micro(acquired_ms) + "\",\"renewTime\":\"" +
         rfc3339_micro(renewed_ms) + "\",\"leaseTransitions\":" + std::to_string(transitions) + "}}";
}

static std::string rv_of(const Json& j) {
  const Json* m = j.get("metadata");
  const Json* rv = m ? m->get("resourceVersion") : nullptr;
  return rv ? rv->str : "";
}

bool KubeLease::acquire(uint64_t& term, std::string& err) {
  bool said_waiting = false;
  for (;;) {
    std::string out;
    const int st = k_.request("GET", path() + "/" + name_, "", out);
    const int64_t now = wall_clock_ms();
    if (st == 404) {
      rv_.clear();
      const int c = k_.request("POST", path(), body(1, now, now), out);
      Json j;
      if ((c == 200 || c == 201) && Json::parse(out, j)) {
        rv_ = rv_of(j);
        term = term_ = 1;
        acquired_ms_ = last_renewed_ms_ = now;
        return true;
      }
      if (c != 409) ES_WARN("lease %s/%s: create answered %d", ns_.c_str(), name_.c_str(), c);
    } else if (st == 200) {
      Json j;
      if (!Json::parse(out, j)) {
        err = "the lease object is not JSON";
        return false;
      }
      const Json* spec = j.get("spec");
      std::string holder;
      int64_t renewed = 0, duration_ms = (int64_t)duration_s_ * 1000;
      uint64_t transitions = 0;
      if (spec) {
        if (const Json* h = spec->get("holderIdentity")) holder = h->str;
        if (const Json* r = spec->get("renewTime")) renewed = parse_rfc3339_ms(r->str);
        if (const Json* d = spec->get("leaseDurationSeconds")) duration_ms = (int64_t)d->num * 1000;
        if (const Json* t = spec->get("leaseTransitions")) transitions = (uint64_t)t->num;
      }
      if (holder.empty() || holder == holder_ || renewed + duration_ms < now) {
        rv_ = rv_of(j);
        const int u = k_.request("PUT", path() + "/" + name_, body(transitions + 1, now, now), out);
        Json uj;
        if (u == 200 && Json::parse(out, uj)) {
          rv_ = rv_of(uj);
          term = term_ = transitions + 1;
          acquired_ms_ = last_renewed_ms_ = now;
          return true;
        }
        if (u != 409) ES_WARN("lease %s/%s: take answered %d", ns_.c_str(), name_.c_str(), u);
        continue;  // another candidate took it first: read it again
      }
      if (!said_waiting) {
        ES_INFO("waiting for the lease %s/%s held by %s", ns_.c_str(), name_.c_str(), holder.c_str());
        said_waiting = true;
      }
    } else {
      ES_WARN("lease %s/%s: the API answered %d", ns_.c_str(), name_.c_str(), st);
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1000));
  }
}

bool KubeLease::renew(std::string& err) {
  const int64_t now = wall_clock_ms();
  std::string out;
  const int u = k_.request("PUT", path() + "/" + name_, body(term_, acquired_ms_, now), out, 2000);
  Json j;
  if (u == 200 && Json::parse(out, j)) {
    rv_ = rv_of(j);
    last_renewed_ms_ = now;
    return true;
  }
  if (u == 409 || u == 200) {
    // someone wrote it since: still ours only if it names this holder and this term
    const int g = k_.request("GET", path() + "/" + name_, "", out, 2000);
    Json gj;
    if (g == 200 && Json::parse(out, gj)) {
      const Json* spec = gj.get("spec");
      const Json* h = spec ? spec->get("holderIdentity") : nullptr;
      const Json* t = spec ? spec->get("leaseTransitions") : nullptr;
      if (!h || h->str != holder_ || !t || (uint64_t)t->num != term_) {
        err = "the lease is held by " + (h ? h->str : std::string("nobody")) + " now";
        return false;
      }
      rv_ = rv_of(gj);
    }
  }
  if (now - last_renewed_ms_ > (int64_t)duration_s_ * 1000) {
    err = "not renewed for " + std::to_string((now - last_renewed_ms_) / 1000) + " s (the API answered " +
          std::to_string(u) + ")";
    return false;
  }
  return true;  // try again at the next period
}

EtcdLease::EtcdLease(std::string url, std::string key, std::string holder, uint32_t ttl_s)
    : url_(std::move(url)), key_(std::move(key)), holder_(std::move(holder)), ca_(env_or("EVERSERVE_ETCD_CA", "")),
      ttl_s_(ttl_s ? ttl_s : 15) {}

int EtcdLease::post(const std::string& path, const std::string& body, std::string& out) const {
  return http_url(url_ + path, "POST", {"Content-Type: application/json"}, body, out, 3000, ca_);
}

// etcd's JSON gateway writes 64-bit numbers as strings
static uint64_t num_of(const Json* j) {
  if (!j) return 0;
  return j->kind == Json::Number ? (uint64_t)j->num : std::strtoull(j->str.c_str(), nullptr, 10);
}

bool EtcdLease::acquire(uint64_t& term, std::string& err) {
  bool said_waiting = false;
  const std::string k64 = base64_encode(key_);
  for (;;) {
    std::string out;
    Json j;
    if (lease_id_.empty()) {
      if (post("/v3/lease/grant", "{\"TTL\":" + std::to_string(ttl_s_) + "}", out) != 200 || !Json::parse(out, j)) {
        ES_WARN("etcd %s: no lease granted", url_.c_str());
        std::this_thread::sleep_for(std::chrono::milliseconds(1000));
        continue;
      }
      const Json* id = j.get("ID");
      lease_id_ = id ? (id->kind == Json::Number ? std::to_string((uint64_t)id->num) : id->str) : "";
      if (lease_id_.empty()) continue;
    }
    // the key is ours only if nobody holds it: created with our lease, or held by someone else
    const std::string txn =
        "{\"compare\":[{\"key\":\"" + k64 + "\",\"result\":\"EQUAL\",\"target\":\"CREATE\",\"create_revision\":\"0\"}],"
        "\"success\":[{\"request_put\":{\"key\":\"" + k64 + "\",\"value\":\"" + base64_encode(holder_) +
        "\",\"lease\":\"" + lease_id_ + "\"}}],\"failure\":[{\"request_range\":{\"key\":\"" + k64 + "\"}}]}";
    if (post("/v3/kv/txn", txn, out) == 200 && Json::parse(out, j)) {
      const Json* ok = j.get("succeeded");
      if (ok && ok->b) {
        const Json* header = j.get("header");
        term = num_of(header ? header->get("revision") : nullptr);  // our key's create revision
        last_renewed_ms_ = wall_clock_ms();
        return term > 0 || (err = "etcd answered no revision", false);
      }
      if (!said_waiting) {
        ES_INFO("waiting for the etcd lease %s", key_.c_str());
        said_waiting = true;
      }
    } else {
      ES_WARN("etcd %s: the transaction was not answered", url_.c_str());
    }
    // keep our own etcd lease alive while we wait, so it is there when the key frees
    post("/v3/lease/keepalive", "{\"ID\":\"" + lease_id_ + "\"}", out);
    std::this_thread::sleep_for(std::chrono::milliseconds(500));
  }
}

bool EtcdLease::renew(std::string& err) {
  std::string out;
  Json j;
  const int64_t now = wall_clock_ms();
  if (post("/v3/lease/keepalive", "{\"ID\":\"" + lease_id_ + "\"}", out) == 200 && Json::parse(out, j)) {
    const Json* res = j.get("result");
    if (!res || num_of(res->get("TTL")) == 0) {
      err = "etcd says the lease expired";
      return false;
    }
    last_renewed_ms_ = now;
    return true;
  }
  if (now - last_renewed_ms_ > (int64_t)ttl_s_ * 1000) {
    err = "not kept alive for " + std::to_string((now - last_renewed_ms_) / 1000) + " s";
    return false;
  }
  return true;
}

}  // namespace es
