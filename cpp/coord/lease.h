// The coordinator's lease: the one process allowed to write epochs. Its term rises with every
// new holder and travels on every message to the daemons, which ignore older terms.
//
//   --lease PATH            a file: an exclusive lock held for the process's life, the term
//                           recorded in the file (one host, or a shared file system with locks)
//   --lease k8s:NS/NAME     a Kubernetes Lease (coordination.k8s.io/v1): held while renewed every
//                           quarter of its duration; `leaseTransitions` is the term; a standby
//                           takes it once the holder's renewTime is older than the duration
//   --lease etcd:URL/KEY    an etcd v3 key (JSON gateway at URL, e.g. http://etcd:2379) created
//                           only if absent, bound to an etcd lease kept alive every quarter of
//                           its TTL; the key's create revision is the term (it grows with every
//                           holder); a standby takes the key once the holder's lease expires
//
// A holder that cannot renew its Kubernetes or etcd lease within the duration has lost it and exits: a
// successor may hold it, and two writers of epochs must never overlap.
//
// Reference parity: controller/src/lease/{mod,file,etcd,kubernetes,renewal}.rs (file lock, etcd
// and Kubernetes Lease with a term, renewal at TTL/4).
#pragma once

#include <cstdint>
#include <memory>
#include <string>

#include "kube.h"

namespace es {

class Lease {
 public:
  virtual ~Lease() = default;
  // Blocks until held; the holder's term.
  virtual bool acquire(uint64_t& term, std::string& err) = 0;
  // One renewal (0 ms period: nothing to renew). False: the lease is lost.
  virtual uint64_t renew_every_ms() const { return 0; }
  virtual bool renew(std::string& err) { return true; }
};

std::unique_ptr<Lease> make_lease(const std::string& spec, const std::string& holder, uint32_t duration_s = 15);

class KubeLease : public Lease {
 public:
  KubeLease(KubeClient k, std::string ns, std::string name, std::string holder, uint32_t duration_s);
  bool acquire(uint64_t& term, std::string& err) override;
  uint64_t renew_every_ms() const override { return duration_s_ * 250ull; }
  bool renew(std::string& err) override;

 private:
  std::string path() const;
  std::string body(uint64_t transitions, int64_t acquired_ms, int64_t renewed_ms) const;
  KubeClient k_;
  std::string ns_, name_, holder_, rv_;
  uint32_t duration_s_;
  uint64_t term_ = 0;
  int64_t acquired_ms_ = 0, last_renewed_ms_ = 0;
};

class EtcdLease : public Lease {
 public:
  EtcdLease(std::string url, std::string key, std::string holder, uint32_t ttl_s);
  bool acquire(uint64_t& term, std::string& err) override;
  uint64_t renew_every_ms() const override { return ttl_s_ * 250ull; }
  bool renew(std::string& err) override;

 private:
  int post(const std::string& path, const std::string& body, std::string& out) const;
  std::string url_, key_, holder_, ca_;
  uint32_t ttl_s_;
  std::string lease_id_;
  int64_t last_renewed_ms_ = 0;
};

}  // namespace es
