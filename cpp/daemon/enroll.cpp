#include "enroll.h"

#include <sys/stat.h>

#include "kube.h"
#include "telemetry.h"
#include "tls.h"
#include "util.h"

namespace es {

bool enrolled_in(const std::string& dir, int64_t margin_ms, Enrolled& out) {
  std::string text, err;
  Json j;
  if (!read_file(dir + "/issued.json", text) || !Json::parse(text, j, &err)) return false;
  const Json* n = j.get("node");
  const Json* na = j.get("notAfterMs");
  const Json* ia = j.get("issuedAtMs");
  if (!n || !na) return false;
  out.node = n->str;
  out.not_after_ms = (int64_t)na->num;
  out.issued_at_ms = ia ? (int64_t)ia->num : 0;
  std::string cert, key;
  return read_file(dir + "/node.crt", cert) && read_file(dir + "/node.key", key) &&
         out.not_after_ms > wall_clock_ms() + margin_ms;
}

bool enroll(const std::string& url, const std::string& dir, const std::string& token_file, Enrolled& out,
            std::string& err) {
  std::string token;
  if (!read_file(token_file, token)) {
    err = "no service-account token at " + token_file;
    return false;
  }
  while (!token.empty() && (token.back() == '\n' || token.back() == '\r' || token.back() == ' ')) token.pop_back();
  std::string key_pem, pub_pem;
  if (!tls::make_key(key_pem, pub_pem, &err)) return false;
  std::string body;
  const int st = http_url(url + "/v1/certificates/node", "POST",
                          {"Authorization: Bearer " + token, "Content-Type: application/json"},
                          "{\"publicKey\":\"" + json_escape(pub_pem) + "\"}", body, 15000, dir + "/ca.crt");
  if (st != 200) {
    err = "the enrollment endpoint answered " + std::to_string(st) + ": " + body.substr(0, 300);
    return false;
  }
  Json j;
  if (!Json::parse(body, j, &err)) return false;
  const Json* node = j.get("node");
  const Json* cert = j.get("certificate");
  const Json* ca = j.get("ca");
  const Json* na = j.get("notAfterMs");
  if (!node || !cert || !ca || !na || cert->str.empty()) {
    err = "the answer lacks the certificate";
    return false;
  }
  mkdirs(dir);
  const int64_t now = wall_clock_ms();
  if (!write_file_atomic(dir + "/node.key", key_pem) || chmod((dir + "/node.key").c_str(), 0600) != 0 ||
      !write_file_atomic(dir + "/node.crt", cert->str) || !write_file_atomic(dir + "/ca.crt", ca->str) ||
      !write_file_atomic(dir + "/issued.json", "{\"node\":\"" + json_escape(node->str) + "\",\"notAfterMs\":" +
                                                   std::to_string((int64_t)na->num) + ",\"issuedAtMs\":" +
                                                   std::to_string(now) + "}")) {
    err = "cannot write into " + dir;
    return false;
  }
  out.node = node->str;
  out.not_after_ms = (int64_t)na->num;
  out.issued_at_ms = now;
  return true;
}

}  // namespace es
