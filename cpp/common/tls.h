// Mutual TLS for the control plane's TCP links (OpenSSL 3, TLS 1.3 only).
//
// Unix sockets stay plain (a node's processes are trusted through the socket directory's
// permissions); every TCP connection between control-plane processes (daemon -> coordinator,
// store -> store replication, operator -> API) is mutually authenticated when TLS is configured:
// both ends present a certificate signed by the cluster's CA, and a peer is known by its
// certificate's common name (a daemon's must be its node's name).
//
// Configuration (each binary reads it at start): EVERSERVE_TLS_DIR plus EVERSERVE_TLS_NAME
// (files ca.crt, <name>.crt, <name>.key in the directory), or EVERSERVE_TLS_CA / _CERT / _KEY.
// `everserve-ctl certs init|issue` makes the CA and the per-process certificates.
#pragma once

#include <cstdint>
#include <string>

#include "net.h"

namespace es {
namespace tls {

struct Config {
  std::string ca, cert, key;
};

bool configure(const Config& c, std::string* err);
// From the environment; true (and TLS off) when nothing is configured.
bool configure_from_env(std::string* err);
// Configure again if a configured file changed since (renewed certificates are taken without a
// restart); false only when the new files do not load (the old ones stay in use).
bool reload_if_changed(std::string* err);
// How often binaries look for changed TLS files: EVERSERVE_TLS_RELOAD_MS, default 30000.
uint64_t reload_period_ms();
bool enabled();

// Non-blocking sessions for the loop (opaque SSL* as void*).
void* new_server(int fd);
void* new_client(int fd);
// 1: done, 0: wants more I/O (`want_write` says which), -1: failed.
int handshake(void* ssl, bool* want_write);
std::string peer_name(void* ssl);
// >0 bytes, 0 closed, -1 would block, -2 error.
long read(void* ssl, char* buf, size_t n);
long write(void* ssl, const char* buf, size_t n);
void free_session(void* ssl);

// A blocking connection for simple clients (CLI, HTTP, store replication): TLS when enabled and
// the address is TCP, plain otherwise.
struct Stream {
  int fd = -1;
  void* ssl = nullptr;
  bool write_all(const std::string& data, int timeout_ms);
  // Reads whatever arrives before `timeout_ms` (at most `n`): >0 bytes, 0 closed, -1 timeout/error.
  long read_some(char* buf, size_t n, int timeout_ms);
  // One frame (4-byte big-endian length + payload) each way.
  bool write_frame(const std::string& payload, int timeout_ms);
  bool read_frame(std::string& payload, int timeout_ms);
  void close();
};
bool connect_stream(const Address& a, int timeout_ms, Stream& out, std::string* err);
// A client connection to a web endpoint outside the cluster's mutual TLS (a cloud metadata
// service, the Kubernetes API): plain TCP, or TLS (1.2 or later) verifying the server against
// `ca_file` (the system's trust store when empty) and the host name asked for.
bool connect_web(const Address& a, bool https, const std::string& ca_file, int timeout_ms, Stream& out,
                 std::string* err);
// The server side of a blocking exchange on an accepted TCP fd (handshake bounded by timeout_ms);
// `client_cert` false: no client certificate is asked (the enrollment endpoint, where a node
// proves itself another way).
bool accept_stream(int fd, int timeout_ms, Stream& out, std::string* err, bool client_cert = true);

// Certificates: a CA (ca.key, ca.crt) and leaf certificates signed by it (<name>.key, <name>.crt,
// CN and DNS name = <name>, IP 127.0.0.1), EC P-256, SHA-256, `days` of validity.
bool make_ca(const std::string& dir, int days, std::string* err);
bool issue(const std::string& dir, const std::string& name, int days, std::string* err);

// Enrollment: a key made where it is used (PEM private key and PEM public key), and a node's
// certificate (CN and DNS name = node, valid `hours`) signed by the CA in `ca_dir` for a public
// key it was sent; also the CA's certificate and the expiry.
bool make_key(std::string& key_pem, std::string& pub_pem, std::string* err);
bool sign_node(const std::string& ca_dir, const std::string& node, const std::string& pub_pem, int hours,
               std::string& cert_pem, std::string& ca_pem, int64_t& not_after_ms, std::string* err);

}  // namespace tls

// sha256 of `data`, lower-case hex.
std::string sha256_hex(const std::string& data);

}  // namespace es
