// everserve-coord-tests: the coordinator's pure functions (fit, degrade, pool placement and codec,
// outcome choice, cover planning). Exits 0 when every check holds; prints each failure.
//
// Reference parity: controller/tests/topology.rs and the policy unit tests of
// controller/src/policy (what they check, in this framework's own cases).
#include <cmath>
#include <cstdio>

#include "cover.h"
#include "everserve_pb.h"
#include "state.h"
#include "topology.h"
#include "util.h"

using namespace es;

static int failures = 0;
#define CHECK(cond)                                                  \
  do {                                                               \
    if (!(cond)) {                                                   \
      std::fprintf(stderr, "%s:%d: CHECK(%s)\n", __FILE__, __LINE__, #cond); \
      failures++;                                                    \
    }                                                                \
  } while (0)

static Device dev(const std::string& node, uint32_t idx, const std::string& cls, uint64_t gib,
                  const std::string& domain = "") {
  Device d;
  d.node = node;
  d.index = idx;
  d.cls = cls;
  d.memory_bytes = gib << 30;
  d.domain = domain.empty() ? node : domain;
  return d;
}

static void test_fit() {
  Position p;
  p.engine = "e0";
  p.cls = "NVIDIA B200";
  p.domain = "rack0";
  // same class, same domain
  Fit f = fit(p, dev("n1", 0, "NVIDIA B200", 180, "rack0"));
  CHECK(f.ok && f.same_class && f.speed == 1.0 && f.same_domain);
  // another domain is reported, not refused
  f = fit(p, dev("n2", 0, "NVIDIA B200", 180, "rack1"));
  CHECK(f.ok && !f.same_domain);
  // a slower class: speed is the bandwidth ratio
  f = fit(p, dev("n1", 1, "NVIDIA H100 80GB HBM3", 80, "rack0"));
  CHECK(f.ok && !f.same_class && std::fabs(f.speed - 3.35 / 8.0) < 1e-9);
  CHECK(f.why.find("in place of") != std::string::npos);
  // a class with no figure: unknown speed
  f = fit(p, dev("n1", 2, "Mystery Accelerator", 64));
  CHECK(f.ok && std::isnan(f.speed));
  // memory decides whether it can hold the position at all
  p.memory_bytes = 100ull << 30;
  f = fit(p, dev("n1", 1, "NVIDIA H100 80GB HBM3", 80));
  CHECK(!f.ok && f.why.find("needs") != std::string::npos);
  // an unknown position class fits any device at speed 1
  Position any;
  f = fit(any, dev("n1", 0, "NVIDIA L4", 24));
  CHECK(f.ok && f.same_class && f.speed == 1.0);
  // most specific names first
  CHECK(class_bandwidth("NVIDIA GB200") == 8.0);
  CHECK(class_bandwidth("NVIDIA H100 PCIe") == 2.0);
  CHECK(class_bandwidth("NVIDIA H100 80GB HBM3") == 3.35);
  CHECK(class_bandwidth("NVIDIA A100-SXM4-40GB") == 1.55);
  CHECK(class_bandwidth("unknown") == 0.0);
}

static void test_degrade() {
  Fit f;
  f.ok = true;
  f.speed = 0.42;  // 58 % slower
  CHECK(within_degrade(f, 0));
  CHECK(within_degrade(f, 60));
  CHECK(!within_degrade(f, 50));
  f.speed = 1.3;  // faster is never a degrade
  CHECK(within_degrade(f, 1));
  f.speed = std::nan("");
  CHECK(within_degrade(f, 0));
  CHECK(!within_degrade(f, 10));
  f.ok = false;
  CHECK(!within_degrade(f, 0));
}

static void test_topology() {
  Topology t;
  t.set_node("n0", {dev("", 0, "NVIDIA B200", 180, ""), dev("", 1, "NVIDIA B200", 180, "")});
  CHECK(t.device("n0", 1) != nullptr && t.device("n0", 1)->node == "n0");
  CHECK(t.domain_of("n0") == "n0");  // no reported domain: the node
  CHECK(t.domain_of("nx") == "nx");
  CHECK(t.device("n0", 5) == nullptr);
  t.remove_node("n0");
  CHECK(t.device("n0", 0) == nullptr);
}

static void test_pools() {
  PoolSpec p;
  std::string err;
  CHECK(parse_pool("{\"name\":\"p0\",\"engines\":[\"a\",\"b\"],\"wants\":3,\"deviceClass\":\"B200\","
                   "\"domain\":\"rack0\",\"command\":[\"x\",\"{pool}\"],\"env\":{\"K\":\"{node}\"},\"generation\":4}",
                   p, err));
  CHECK(p.name == "p0" && p.engines.size() == 2 && p.wants == 3 && p.device_class == "B200" && p.domain == "rack0");
  CHECK(p.command.size() == 2 && p.env["K"] == "{node}" && p.generation == 4);
  PoolSpec q;
  CHECK(parse_pool(pool_json(p), q, err));  // the codec round-trips
  CHECK(q.name == p.name && q.engines == p.engines && q.wants == p.wants && q.env == p.env && q.generation == 4);
  CHECK(!parse_pool("[1]", q, err));

  std::vector<FreeDevice> free = {{"n0", 2, "NVIDIA B200", "rack0"}, {"n0", 3, "NVIDIA B200", "rack0"},
                                  {"n1", 0, "NVIDIA B200", "rack0"}, {"n2", 0, "NVIDIA B200", "rack1"},
                                  {"n3", 0, "NVIDIA H100 80GB HBM3", "rack0"}};
  auto got = place_pool_spares(p, free, 3);  // class and domain filter, spread over nodes
  CHECK(got.size() == 3);
  CHECK(got[0] == std::make_pair(std::string("n0"), 2u));
  CHECK(got[1] == std::make_pair(std::string("n1"), 0u));
  CHECK(got[2] == std::make_pair(std::string("n0"), 3u));
  p.domain.clear();
  p.device_class = "H100";
  got = place_pool_spares(p, free, 5);
  CHECK(got.size() == 1 && got[0].first == "n3");
  p.device_class.clear();
  CHECK(place_pool_spares(p, free, 0).empty());
}

static void test_policy_and_outcome() {
  Policy pol;
  std::string err;
  CHECK(parse_policy("{\"outcomesInOrder\":[\"OUTCOME_REPLACE\",\"OUTCOME_SHRINK\"],"
                     "\"spares\":{\"perEngine\":2,\"loading\":\"LOADING_ON_NOTICE\",\"allowMismatched\":true,"
                     "\"maxDegradePercent\":40},"
                     "\"engines\":[{\"name\":\"e0\",\"tensorParallel\":4,\"placementIndependentModel\":true}]}",
                     pol, err));
  CHECK(pol.spares.per_engine == 2 && pol.spares.loading == 2 && pol.spares.allow_mismatched &&
        pol.spares.max_degrade_percent == 40);
  CHECK(pol.world_size("e0") == 4);
  std::vector<SpareSeat> seats(2);
  seats[0].node = "n1";
  seats[0].for_rank = -1;
  seats[1].node = "n2";
  seats[1].for_rank = 2;
  // its own rank's spare first, then an any-rank spare
  Choice c = choose_outcome(pol, "e0", {2, 3}, seats);
  CHECK(c.outcome == signals::Outcome_OUTCOME_REPLACE && c.take.size() == 2);
  CHECK(c.take[0].first == 2 && c.take[0].second.node == "n2");
  CHECK(c.take[1].first == 3 && c.take[1].second.node == "n1");
  // three losses, two spares: SHRINK (placement independent)
  c = choose_outcome(pol, "e0", {1, 2, 3}, seats);
  CHECK(c.outcome == signals::Outcome_OUTCOME_SHRINK);
  // another build cannot take a rank
  seats[0].fingerprint = "other";
  seats[1].fingerprint = "other";
  c = choose_outcome(pol, "e0", {2}, seats, "mine");
  CHECK(c.outcome == signals::Outcome_OUTCOME_SHRINK);
}

int main() {
  test_fit();
  test_degrade();
  test_topology();
  test_pools();
  test_policy_and_outcome();
  if (failures) {
    std::fprintf(stderr, "%d check(s) failed\n", failures);
    return 1;
  }
  std::printf("all checks passed\n");
  return 0;
}
