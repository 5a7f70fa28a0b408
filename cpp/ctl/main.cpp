// everserve-ctl: the operator's client of the coordinator's REST API.
//
//   everserve-ctl [--api host:port] get engines|nodes|pools|engine NAME|pool NAME
//   everserve-ctl [--api host:port] pool apply NAME FILE [--generation N] | pool delete NAME
//   everserve-ctl [--api host:port] watch [--since N] [--once]
//   everserve-ctl [--api host:port] cordon|uncordon|drain|undrain NODE
//   everserve-ctl [--api host:port] stacks ENGINE
//   everserve-ctl [--api host:port] events ENGINE
//   everserve-ctl [--api host:port] openapi
//   everserve-ctl check [--policy FILE]
//   everserve-ctl certs init DIR | certs issue DIR NAME   (the cluster CA and per-process certificates)
// The API address also comes from EVERSERVE_API_ADDR. Subcommands follow the reference CLI's
// operator verbs (controller/src/cli/*.rs; controller/README.md:100-115).
#include <unistd.h>

#include <cstdio>
#include <string>
#include <vector>

#include "../coord/state.h"
#include "telemetry.h"
#include "tls.h"
#include "util.h"

using namespace es;

static int usage() {
  fprintf(stderr,
          "usage: everserve-ctl [--api ADDR] get engines|nodes|pools|engine NAME|pool NAME\n"
          "       everserve-ctl [--api ADDR] pool apply NAME FILE [--generation N] | pool delete NAME\n"
          "       everserve-ctl [--api ADDR] watch [--since N] [--once]\n"
          "       everserve-ctl [--api ADDR] cordon|uncordon|drain|undrain NODE\n"
          "       everserve-ctl [--api ADDR] stacks ENGINE\n"
          "       everserve-ctl [--api ADDR] events ENGINE\n"
          "       everserve-ctl [--api ADDR] openapi\n"
          "       everserve-ctl check --policy FILE\n"
          "       everserve-ctl certs init DIR [--days N] | certs issue DIR NAME [--days N]\n");
  return 2;
}

static int call(const std::string& api, const std::string& method, const std::string& path,
                const std::string& body = "") {
  std::string out;
  const int code = http_request(api, method, path, body, out);
  if (code < 0) {
    fprintf(stderr, "cannot reach the coordinator at %s\n", api.c_str());
    return 1;
  }
  printf("%s\n", out.c_str());
  return code == 200 ? 0 : 1;
}

int main(int argc, char** argv) {
  {
    std::string terr;
    if (!es::tls::configure_from_env(&terr)) {
      fprintf(stderr, "TLS: %s\n", terr.c_str());
      return 2;
    }
  }
  std::string api = env_or("EVERSERVE_API_ADDR", "127.0.0.1:7681");
  std::vector<std::string> args;
  for (int i = 1; i < argc; i++) {
    const std::string a = argv[i];
    if (a == "--api" && i + 1 < argc) api = argv[++i];
    else args.push_back(a);
  }
  if (args.empty()) return usage();
  const std::string& verb = args[0];
  if (verb == "pool") {
    // a pool's spec (spec.v1.PoolSpec as proto3 JSON) written over the generation held, or only
    // over `--generation N` when given
    if (args.size() >= 3 && args[1] == "delete") return call(api, "DELETE", "/v1/pools/" + args[2]);
    if (args.size() >= 4 && args[1] == "apply") {
      std::string body;
      if (!read_file(args[3], body)) {
        fprintf(stderr, "cannot read %s\n", args[3].c_str());
        return 1;
      }
      std::string path = "/v1/pools/" + args[2];
      if (args.size() >= 6 && args[4] == "--generation") path += "?generation=" + args[5];
      return call(api, "PUT", path, body);
    }
    return usage();
  }
  if (verb == "get") {
    if (args.size() >= 2 && (args[1] == "engines" || args[1] == "nodes" || args[1] == "pools"))
      return call(api, "GET", "/v1/" + args[1]);
    if (args.size() >= 3 && args[1] == "engine") return call(api, "GET", "/v1/engines/" + args[2]);
    if (args.size() >= 3 && args[1] == "pool") return call(api, "GET", "/v1/pools/" + args[2]);
    return usage();
  }
  if (verb == "cordon" || verb == "uncordon" || verb == "drain" || verb == "undrain") {
    if (args.size() < 2) return usage();
    return call(api, "PUT", "/v1/nodes/" + args[1] + "/" + verb);
  }
  if (verb == "events") {
    if (args.size() < 2) return usage();
    return call(api, "GET", "/v1/engines/" + args[1] + "/events");
  }
  if (verb == "stacks") {
    if (args.size() < 2) return usage();
    return call(api, "POST", "/v1/engines/" + args[1] + "/stacks");
  }
  if (verb == "openapi") return call(api, "GET", "/v1/openapi");
  if (verb == "watch") {
    uint64_t since = 0;
    bool once = false;
    for (size_t i = 1; i < args.size(); i++) {
      if (args[i] == "--since" && i + 1 < args.size()) since = std::stoull(args[++i]);
      else if (args[i] == "--once") once = true;
    }
    for (;;) {
      std::string out;
      if (http_request(api, "GET", "/v1/watch?since=" + std::to_string(since), "", out) != 200) {
        fprintf(stderr, "cannot reach the coordinator at %s\n", api.c_str());
        return 1;
      }
      Json j;
      std::string err;
      if (Json::parse(out, j, &err))
        if (const Json* evs = j.get("events"))
          for (auto& ev : evs->arr) {
            const Json* seq = ev.get("seq");
            const Json* text = ev.get("text");
            if (seq) since = (uint64_t)seq->num;
            printf("%llu %s\n", (unsigned long long)since, text ? text->str.c_str() : "");
          }
      fflush(stdout);
      if (once) return 0;
      usleep(500 * 1000);
    }
  }
  if (verb == "certs") {
    // certs init DIR [--days N] | certs issue DIR NAME [--days N]
    int days = 365;
    for (size_t i = 1; i + 1 < args.size(); i++)
      if (args[i] == "--days") days = std::stoi(args[i + 1]);
    std::string err;
    if (args.size() >= 3 && args[1] == "init") {
      if (!tls::make_ca(args[2], days, &err)) {
        fprintf(stderr, "%s\n", err.c_str());
        return 1;
      }
      printf("CA written to %s (ca.key, ca.crt)\n", args[2].c_str());
      return 0;
    }
    if (args.size() >= 4 && args[1] == "issue") {
      if (!tls::issue(args[2], args[3], days, &err)) {
        fprintf(stderr, "%s\n", err.c_str());
        return 1;
      }
      printf("certificate for %s written to %s\n", args[3].c_str(), args[2].c_str());
      return 0;
    }
    return usage();
  }
  if (verb == "check") {
    std::string path;
    for (size_t i = 1; i + 1 < args.size(); i++)
      if (args[i] == "--policy") path = args[i + 1];
    if (path.empty()) return usage();
    std::string text, err;
    Policy p;
    if (!read_file(path, text) || !parse_policy(text, p, err)) {
      printf("policy %s: INVALID: %s\n", path.c_str(), err.empty() ? "unreadable" : err.c_str());
      return 1;
    }
    printf("policy %s: ok (%zu engine(s), %zu outcome(s))\n", path.c_str(), p.engines.size(), p.outcomes.size());
    for (auto& [name, e] : p.engines)
      printf("  engine %s: tp %u pp %u dp %u ep %u, world %u\n", name.c_str(), e.tensor, e.pipeline, e.data, e.expert,
             p.world_size(name));
    return 0;
  }
  return usage();
}
