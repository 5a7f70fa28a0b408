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

// ---- cover planning --------------------------------------------------------------------------
static SpareSeat seat(const std::string& node, uint32_t device, int64_t for_rank) {
  SpareSeat s;
  s.node = node;
  s.device = device;
  s.for_rank = for_rank;
  return s;
}

static CoverInput cover_in(uint32_t tp, uint32_t pp, const std::vector<std::pair<std::string, std::vector<uint32_t>>>& nodes) {
  CoverInput in;
  in.engine = "e0";
  in.tp = tp;
  in.pp = pp;
  for (auto& [node, ranks] : nodes)
    for (uint32_t r : ranks) in.holders[r] = {node, r};
  return in;
}

static std::vector<std::string> purposes(const signals::CoverPlan& p) {
  std::vector<std::string> out;
  for (auto& s : p.sets) out.push_back(s.purpose);
  return out;
}

static void test_cover() {
  // TP1 PP2 over two nodes with one any-rank spare on a third node
  CoverInput in = cover_in(1, 2, {{"a", {0}}, {"b", {1}}});
  in.spares = {seat("c", 0, -1)};
  std::vector<std::vector<uint32_t>> covers;
  std::vector<Uncovered> unc;
  auto plan = plan_cover(in, &covers, &unc);
  auto ps = purposes(plan);
  // the current set, then each node's loss (each node holds one rank here, so no position losses)
  CHECK(ps.size() == 3 && ps[0] == "current" && ps[1] == "REPLACE of ranks [0]" && ps[2] == "REPLACE of ranks [1]");
  CHECK(covers.size() == 3 && covers[0].empty() && covers[1] == std::vector<uint32_t>{0});
  CHECK(unc.empty());
  CHECK(plan.sets[1].members[0].has_spare && plan.sets[1].members[0].spare.node == "c" && !plan.sets[1].members[1].has_spare);
  // one pipeline group per set, the current set's group first and shared by no other set
  CHECK(plan.groups.size() == 3 && plan.sets[0].groups.size() == 1);

  // TP2 PP1 on one node with two any-rank spares on another: the node's loss needs both spares,
  // then each position's loss; second spares after every first cover
  in = cover_in(2, 1, {{"a", {0, 1}}});
  in.spares = {seat("s", 0, -1), seat("s", 1, -1)};
  covers.clear();
  unc.clear();
  plan = plan_cover(in, &covers, &unc);
  ps = purposes(plan);
  CHECK(ps.size() == 6);
  CHECK(ps[1] == "REPLACE of ranks [0, 1]" && ps[2] == "REPLACE of ranks [0]" && ps[3] == "REPLACE of ranks [1]");
  CHECK(ps[4] == "REPLACE of ranks [0] through a second spare" && ps[5] == "REPLACE of ranks [1] through a second spare");
  CHECK(answers(plan.sets[1].members, {0, 1}) && answers(plan.sets[2].members, {0}) && !answers(plan.sets[2].members, {1}));
  // the second spare is another seat than the first
  CHECK(plan.sets[4].members[0].spare.device != plan.sets[2].members[0].spare.device);
  CHECK(unc.empty());

  // a spare on the lost node dies with it: the node's loss is uncovered, its positions are not
  in = cover_in(2, 1, {{"a", {0, 1}}});
  in.spares = {seat("a", 5, -1)};
  unc.clear();
  plan = plan_cover(in, nullptr, &unc);
  CHECK(unc.size() == 1 && unc[0].lost == (std::vector<uint32_t>{0, 1}) && unc[0].why.find("no spare") != std::string::npos);

  // SHRINK allowed: every loss also gets its survivors' set
  in = cover_in(2, 1, {{"a", {0}}, {"b", {1}}});
  in.replace = false;
  in.shrink = true;
  plan = plan_cover(in);
  ps = purposes(plan);
  CHECK(ps.size() == 3 && ps[1] == "SHRINK of ranks [0]" && plan.sets[1].members.size() == 1);

  // neither outcome: every loss uncovered with the policy as the reason
  in.shrink = false;
  unc.clear();
  plan_cover(in, nullptr, &unc);
  CHECK(unc.size() == 2 && unc[0].why.find("neither") != std::string::npos);

  // the budget bounds the groups a process holds (TP1 PP2: each set needs one group over both
  // members); the sets it refuses are reported as over the budget
  in = cover_in(1, 2, {{"a", {0}}, {"b", {1}}});
  in.spares = {seat("c", 0, -1)};
  in.max_groups_per_gpu = 2;  // the current group plus one more each: both replacement sets fit
  unc.clear();
  plan = plan_cover(in, nullptr, &unc);
  CHECK(plan.sets.size() == 3 && unc.empty());
  in.max_groups_per_gpu = 1;  // the current group only
  unc.clear();
  plan = plan_cover(in, nullptr, &unc);
  CHECK(plan.sets.size() == 1 && unc.size() == 2 && unc[0].why.find("budget of 1") != std::string::npos);
  // groups other engines' plans put on the spare count too
  in.max_groups_per_gpu = 3;
  in.elsewhere[{"c", 0}] = 3;
  unc.clear();
  plan = plan_cover(in, nullptr, &unc);
  CHECK(plan.sets.size() == 1 && unc.size() == 2);

  // a spare for rank 1 takes rank 1 ahead of an any-rank spare
  in = cover_in(2, 1, {{"a", {0}}, {"b", {1}}});
  in.spares = {seat("x", 0, -1), seat("y", 0, 1)};
  plan = plan_cover(in);
  for (auto& st : plan.sets)
    if (st.purpose == "REPLACE of ranks [1]") CHECK(st.members[1].spare.node == "y");
}

int main() {
  test_cover();
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
