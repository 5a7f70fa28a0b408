// A node daemon's side of enrollment (the coordinator's issuer.h): a key made here and never
// sent, its public half and the pod's projected service-account token sent to the coordinator's
// enrollment endpoint, and the certificate it answers with, for the node the API server says the
// pod runs on. Written to one directory, each file replaced in one step: node.key (0600),
// node.crt, ca.crt, and last issued.json ({"node", "notAfterMs", "issuedAtMs"}), so issued.json
// never says more than the files hold. The daemon renews at half the certificate's life.
//
// The endpoint is verified against the bootstrap CA (ca.crt already in the directory, e.g. from
// a ConfigMap); the token comes from EVERSERVE_ENROLL_TOKEN_FILE (default
// /var/run/secrets/everserve/token).
#pragma once

#include <cstdint>
#include <string>

namespace es {

struct Enrolled {
  std::string node;
  int64_t not_after_ms = 0, issued_at_ms = 0;
};

// The certificate already in `dir`, if issued.json says it is valid for at least `margin_ms`.
bool enrolled_in(const std::string& dir, int64_t margin_ms, Enrolled& out);
// One enrollment: writes the files; false with `err` when refused or unreachable.
bool enroll(const std::string& url, const std::string& dir, const std::string& token_file, Enrolled& out,
            std::string& err);

}  // namespace es
