// everserve-codec-check: the generated protobuf codec (gen/everserve_pb.h) and the policy parser
// driven from standard input, for tests that compare them with other encoders.
//
//   <full message name> <hex bytes>   ->  the codec's decode then encode, as hex ("ERR" if refused)
//   policy <hex of proto3 JSON text>  ->  the coordinator's reading of that policy, one line of JSON
#include <cstdio>
#include <iostream>
#include <string>

#include "../coord/state.h"
#include "everserve_pb.h"

static std::string from_hex(const std::string& h) {
  std::string out;
  for (size_t i = 0; i + 1 < h.size(); i += 2) out.push_back((char)std::stoi(h.substr(i, 2), nullptr, 16));
  return out;
}

static std::string to_hex(const std::string& b) {
  static const char* d = "0123456789abcdef";
  std::string out;
  for (unsigned char c : b) {
    out.push_back(d[c >> 4]);
    out.push_back(d[c & 15]);
  }
  return out;
}

static std::string policy_summary(const es::Policy& p) {
  std::string s = "{\"outcomes\":[";
  for (size_t i = 0; i < p.outcomes.size(); i++) s += (i ? "," : "") + std::to_string(p.outcomes[i]);
  s += "],\"maxConcurrentLosses\":" + std::to_string(p.max_concurrent_losses) +
       ",\"coverEnabled\":" + (p.cover_enabled ? "true" : "false") +
       ",\"coverMaxGroupsPerGpu\":" + std::to_string(p.cover_max_groups_per_gpu) + ",\"engines\":{";
  bool first = true;
  for (auto& [name, e] : p.engines) {
    s += std::string(first ? "" : ",") + "\"" + name + "\":{\"tp\":" + std::to_string(e.tensor) +
         ",\"pp\":" + std::to_string(e.pipeline) + ",\"dp\":" + std::to_string(e.data) +
         ",\"placementIndependent\":" + (e.placement_independent ? "true" : "false") + "}";
    first = false;
  }
  return s + "}}";
}

int main() {
  std::string line;
  while (std::getline(std::cin, line)) {
    const size_t sp = line.find(' ');
    if (sp == std::string::npos) {
      std::cout << "ERR\n";
      continue;
    }
    const std::string name = line.substr(0, sp), body = from_hex(line.substr(sp + 1));
    if (name == "policy") {
      es::Policy p;
      std::string err;
      std::cout << (es::parse_policy(body, p, err) ? policy_summary(p) : "ERR " + err) << "\n";
      continue;
    }
    std::string out;
    std::cout << (pbgen::roundtrip(name, body, out) ? to_hex(out) : "ERR") << "\n";
  }
  return 0;
}
