#include "tls.h"

#include <openssl/err.h>
#include <openssl/evp.h>
#include <openssl/pem.h>
#include <openssl/ssl.h>
#include <openssl/x509v3.h>
#include <arpa/inet.h>
#include <poll.h>
#include <sys/stat.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <cstdio>
#include <cstdlib>
#include <ctime>

#include "util.h"

namespace es {
namespace tls {
namespace {

SSL_CTX* g_server = nullptr;
SSL_CTX* g_client = nullptr;
SSL_CTX* g_server_open = nullptr;  // the same identity, no client certificate asked (enrollment)
// the contexts are replaced when the files change (reload_if_changed): a session is made under
// this lock, and holds its own reference to its context from then on
std::mutex g_mu;
Config g_config;
std::map<std::string, long long> g_mtimes;

long long mtime_of(const std::string& path) {
  struct stat st;
  if (stat(path.c_str(), &st) != 0) return -1;
  return (long long)st.st_mtim.tv_sec * 1000000000ll + st.st_mtim.tv_nsec;
}

std::string last_error() {
  char buf[256];
  ERR_error_string_n(ERR_get_error(), buf, sizeof(buf));
  return buf;
}

SSL_CTX* make_ctx(bool server, const Config& c, std::string* err) {
  SSL_CTX* ctx = SSL_CTX_new(server ? TLS_server_method() : TLS_client_method());
  if (!ctx) {
    if (err) *err = "SSL_CTX_new: " + last_error();
    return nullptr;
  }
  SSL_CTX_set_min_proto_version(ctx, TLS1_3_VERSION);
  SSL_CTX_set_mode(ctx, SSL_MODE_ENABLE_PARTIAL_WRITE | SSL_MODE_ACCEPT_MOVING_WRITE_BUFFER);
  if (SSL_CTX_use_certificate_chain_file(ctx, c.cert.c_str()) != 1 ||
      SSL_CTX_use_PrivateKey_file(ctx, c.key.c_str(), SSL_FILETYPE_PEM) != 1 || SSL_CTX_check_private_key(ctx) != 1 ||
      SSL_CTX_load_verify_locations(ctx, c.ca.c_str(), nullptr) != 1) {
    if (err) *err = "TLS files (" + c.cert + ", " + c.key + ", " + c.ca + "): " + last_error();
    SSL_CTX_free(ctx);
    return nullptr;
  }
  SSL_CTX_set_verify(ctx, SSL_VERIFY_PEER | SSL_VERIFY_FAIL_IF_NO_PEER_CERT, nullptr);
  return ctx;
}

bool wait_fd(int fd, bool write, int timeout_ms) {
  pollfd pf{fd, (short)(write ? POLLOUT : POLLIN), 0};
  return ::poll(&pf, 1, timeout_ms) > 0;
}

}  // namespace

bool configure(const Config& c, std::string* err) {
  SSL_CTX* server = make_ctx(true, c, err);
  if (!server) return false;
  SSL_CTX* client = make_ctx(false, c, err);
  SSL_CTX* open = make_ctx(true, c, err);
  if (!client || !open) {
    SSL_CTX_free(server);
    if (client) SSL_CTX_free(client);
    return false;
  }
  SSL_CTX_set_verify(open, SSL_VERIFY_NONE, nullptr);
  // replaced contexts are freed: sessions made from them hold their own references
  {
    std::lock_guard<std::mutex> g(g_mu);
    std::swap(g_server, server);
    std::swap(g_client, client);
    std::swap(g_server_open, open);
    g_config = c;
    g_mtimes.clear();
    for (auto* f : {&c.ca, &c.cert, &c.key}) g_mtimes[*f] = mtime_of(*f);
  }
  for (SSL_CTX* old : {server, client, open})
    if (old) SSL_CTX_free(old);
  return true;
}

uint64_t reload_period_ms() {
  static const uint64_t ms = std::strtoull(env_or("EVERSERVE_TLS_RELOAD_MS", "30000").c_str(), nullptr, 10);
  return ms ? ms : 30000;
}

bool reload_if_changed(std::string* err) {
  Config c;
  bool changed = false;
  {
    std::lock_guard<std::mutex> g(g_mu);
    if (g_server == nullptr) return true;
    c = g_config;
    for (auto& [f, t] : g_mtimes) changed |= mtime_of(f) != t;
  }
  if (!changed) return true;
  if (!configure(c, err)) return false;
  ES_INFO("TLS files changed: certificates reloaded");
  return true;
}

bool configure_from_env(std::string* err) {
  Config c;
  const std::string dir = env_or("EVERSERVE_TLS_DIR", "");
  if (!dir.empty()) {
    const std::string name = env_or("EVERSERVE_TLS_NAME", "");
    if (name.empty()) {
      if (err) *err = "EVERSERVE_TLS_DIR needs EVERSERVE_TLS_NAME";
      return false;
    }
    c.ca = dir + "/ca.crt";
    c.cert = dir + "/" + name + ".crt";
    c.key = dir + "/" + name + ".key";
  } else {
    c.ca = env_or("EVERSERVE_TLS_CA", "");
    c.cert = env_or("EVERSERVE_TLS_CERT", "");
    c.key = env_or("EVERSERVE_TLS_KEY", "");
    if (c.ca.empty() && c.cert.empty() && c.key.empty()) return true;  // TLS off
  }
  return configure(c, err);
}

bool enabled() { return g_server != nullptr && g_client != nullptr; }

void* new_server(int fd) {
  std::lock_guard<std::mutex> g(g_mu);
  SSL* s = SSL_new(g_server);
  SSL_set_fd(s, fd);
  SSL_set_accept_state(s);
  return s;
}

void* new_client(int fd) {
  std::lock_guard<std::mutex> g(g_mu);
  SSL* s = SSL_new(g_client);
  SSL_set_fd(s, fd);
  SSL_set_connect_state(s);
  return s;
}

int handshake(void* p, bool* want_write) {
  SSL* s = static_cast<SSL*>(p);
  const int r = SSL_do_handshake(s);
  if (r == 1) return 1;
  const int e = SSL_get_error(s, r);
  if (e == SSL_ERROR_WANT_READ || e == SSL_ERROR_WANT_WRITE) {
    if (want_write) *want_write = e == SSL_ERROR_WANT_WRITE;
    return 0;
  }
  ERR_clear_error();
  return -1;
}

std::string peer_name(void* p) {
  X509* x = SSL_get1_peer_certificate(static_cast<SSL*>(p));
  if (!x) return "";
  char buf[256] = {0};
  X509_NAME_get_text_by_NID(X509_get_subject_name(x), NID_commonName, buf, sizeof(buf) - 1);
  X509_free(x);
  return buf;
}

long read(void* p, char* buf, size_t n) {
  SSL* s = static_cast<SSL*>(p);
  const int r = SSL_read(s, buf, (int)n);
  if (r > 0) return r;
  const int e = SSL_get_error(s, r);
  if (e == SSL_ERROR_WANT_READ || e == SSL_ERROR_WANT_WRITE) return -1;
  if (e == SSL_ERROR_ZERO_RETURN) return 0;
  ERR_clear_error();
  return -2;
}

long write(void* p, const char* buf, size_t n) {
  SSL* s = static_cast<SSL*>(p);
  const int r = SSL_write(s, buf, (int)n);
  if (r > 0) return r;
  const int e = SSL_get_error(s, r);
  if (e == SSL_ERROR_WANT_READ || e == SSL_ERROR_WANT_WRITE) return -1;
  ERR_clear_error();
  return -2;
}

void free_session(void* p) {
  if (p) SSL_free(static_cast<SSL*>(p));
}

// ---- blocking streams ------------------------------------------------------------------------
static bool finish_handshake(Stream& s, int timeout_ms, std::string* err) {
  const uint64_t deadline = now_ms() + (uint64_t)timeout_ms;
  while (true) {
    bool ww = false;
    const int r = handshake(s.ssl, &ww);
    if (r == 1) return true;
    if (r < 0 || now_ms() >= deadline || !wait_fd(s.fd, ww, (int)(deadline - now_ms()))) {
      if (err) *err = "TLS handshake failed";
      return false;
    }
  }
}

bool connect_stream(const Address& a, int timeout_ms, Stream& out, std::string* err) {
  out = Stream{};
  out.fd = connect_to(a, timeout_ms, err);
  if (out.fd < 0) return false;
  if (!a.unix_socket && enabled()) {
    out.ssl = new_client(out.fd);
    if (!finish_handshake(out, timeout_ms, err)) {
      out.close();
      return false;
    }
  }
  return true;
}

bool connect_web(const Address& a, bool https, const std::string& ca_file, int timeout_ms, Stream& out,
                 std::string* err) {
  out = Stream{};
  out.fd = connect_to(a, timeout_ms, err);
  if (out.fd < 0) return false;
  if (!https) return true;
  // one client context per CA file (the system's trust store for ""), made on first use
  static std::mutex mu;
  static std::map<std::string, SSL_CTX*> ctxs;
  SSL_CTX* ctx = nullptr;
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = ctxs.find(ca_file);
    if (it != ctxs.end()) {
      ctx = it->second;
    } else {
      ctx = SSL_CTX_new(TLS_client_method());
      if (ctx) {
        SSL_CTX_set_min_proto_version(ctx, TLS1_2_VERSION);
        SSL_CTX_set_mode(ctx, SSL_MODE_ENABLE_PARTIAL_WRITE | SSL_MODE_ACCEPT_MOVING_WRITE_BUFFER);
        const int ok = ca_file.empty() ? SSL_CTX_set_default_verify_paths(ctx)
                                       : SSL_CTX_load_verify_locations(ctx, ca_file.c_str(), nullptr);
        if (ok != 1) {
          if (err) *err = "CA " + (ca_file.empty() ? std::string("(system)") : ca_file) + ": " + last_error();
          SSL_CTX_free(ctx);
          ctx = nullptr;
        } else {
          SSL_CTX_set_verify(ctx, SSL_VERIFY_PEER, nullptr);
          ctxs[ca_file] = ctx;
        }
      }
    }
  }
  if (!ctx) {
    out.close();
    return false;
  }
  SSL* s = SSL_new(ctx);
  SSL_set_fd(s, out.fd);
  SSL_set_connect_state(s);
  // the certificate must name the host (or the IP address) asked for
  in6_addr ip6;
  in_addr ip4;
  if (inet_pton(AF_INET, a.host.c_str(), &ip4) == 1 || inet_pton(AF_INET6, a.host.c_str(), &ip6) == 1) {
    X509_VERIFY_PARAM_set1_ip_asc(SSL_get0_param(s), a.host.c_str());
  } else {
    SSL_set_tlsext_host_name(s, a.host.c_str());
    SSL_set1_host(s, a.host.c_str());
  }
  out.ssl = s;
  if (!finish_handshake(out, timeout_ms, err)) {
    out.close();
    return false;
  }
  return true;
}

bool accept_stream(int fd, int timeout_ms, Stream& out, std::string* err, bool client_cert) {
  out = Stream{};
  out.fd = fd;
  if (enabled()) {
    if (client_cert) {
      out.ssl = new_server(fd);
    } else {
      std::lock_guard<std::mutex> g(g_mu);
      SSL* s = SSL_new(g_server_open);
      SSL_set_fd(s, fd);
      SSL_set_accept_state(s);
      out.ssl = s;
    }
    if (!finish_handshake(out, timeout_ms, err)) {
      out.close();
      return false;
    }
  }
  return true;
}

bool Stream::write_all(const std::string& data, int timeout_ms) {
  const uint64_t deadline = now_ms() + (uint64_t)timeout_ms;
  size_t off = 0;
  while (off < data.size()) {
    long w;
    if (ssl) {
      w = write(ssl, data.data() + off, data.size() - off);
      if (w == -2) return false;
    } else {
      w = ::send(fd, data.data() + off, data.size() - off, MSG_NOSIGNAL);
      if (w < 0 && errno != EAGAIN && errno != EINTR) return false;
      if (w < 0) w = -1;
    }
    if (w > 0) {
      off += (size_t)w;
      continue;
    }
    if (now_ms() >= deadline || !wait_fd(fd, true, (int)(deadline - now_ms()))) return false;
  }
  return true;
}

long Stream::read_some(char* buf, size_t n, int timeout_ms) {
  const uint64_t deadline = now_ms() + (uint64_t)timeout_ms;
  while (true) {
    long r;
    if (ssl) {
      r = read(ssl, buf, n);
      if (r == -2) return -1;
    } else {
      r = ::recv(fd, buf, n, MSG_DONTWAIT);
      if (r < 0 && errno != EAGAIN && errno != EINTR) return -1;
      if (r < 0) r = -1;
    }
    if (r >= 0) return r;
    if (now_ms() >= deadline || !wait_fd(fd, false, (int)(deadline - now_ms()))) return -1;
  }
}

bool Stream::write_frame(const std::string& payload, int timeout_ms) {
  std::string out;
  if (!encode_frame(payload, out)) return false;
  return write_all(out, timeout_ms);
}

bool Stream::read_frame(std::string& payload, int timeout_ms) {
  const uint64_t deadline = now_ms() + (uint64_t)timeout_ms;
  auto exact = [&](char* dst, size_t n) {
    size_t got = 0;
    while (got < n) {
      const int left = (int)std::max<int64_t>(1, (int64_t)deadline - (int64_t)now_ms());
      const long r = read_some(dst + got, n - got, left);
      if (r <= 0) return false;
      got += (size_t)r;
    }
    return true;
  };
  unsigned char h[4];
  if (!exact(reinterpret_cast<char*>(h), 4)) return false;
  const uint32_t n = (uint32_t)h[0] << 24 | (uint32_t)h[1] << 16 | (uint32_t)h[2] << 8 | h[3];
  if (n > kMaxFrame) return false;
  payload.resize(n);
  return n == 0 || exact(payload.data(), n);
}

void Stream::close() {
  if (ssl) {
    SSL_shutdown(static_cast<SSL*>(ssl));
    free_session(ssl);
    ssl = nullptr;
  }
  if (fd >= 0) ::close(fd);
  fd = -1;
}

// ---- certificates ----------------------------------------------------------------------------
static bool write_pem(const std::string& path, EVP_PKEY* key, X509* cert) {
  FILE* f = fopen(path.c_str(), "w");
  if (!f) return false;
  const bool ok = key ? PEM_write_PrivateKey(f, key, nullptr, nullptr, 0, nullptr, nullptr) == 1
                      : PEM_write_X509(f, cert) == 1;
  fclose(f);
  if (key) chmod(path.c_str(), 0600);
  return ok;
}

static bool add_ext(X509* cert, X509* issuer, int nid, const char* value) {
  X509V3_CTX ctx;
  X509V3_set_ctx_nodb(&ctx);
  X509V3_set_ctx(&ctx, issuer, cert, nullptr, nullptr, 0);
  X509_EXTENSION* ext = X509V3_EXT_conf_nid(nullptr, &ctx, nid, value);
  if (!ext) return false;
  X509_add_ext(cert, ext, -1);
  X509_EXTENSION_free(ext);
  return true;
}

static X509* new_cert(EVP_PKEY* key, const std::string& cn, int days, long serial) {
  X509* x = X509_new();
  X509_set_version(x, 2);
  ASN1_INTEGER_set(X509_get_serialNumber(x), serial);
  X509_gmtime_adj(X509_getm_notBefore(x), -60);
  X509_gmtime_adj(X509_getm_notAfter(x), (long)days * 86400);
  X509_set_pubkey(x, key);
  X509_NAME_add_entry_by_txt(X509_get_subject_name(x), "CN", MBSTRING_ASC,
                             reinterpret_cast<const unsigned char*>(cn.c_str()), -1, -1, 0);
  return x;
}

bool make_ca(const std::string& dir, int days, std::string* err) {
  mkdirs(dir);
  EVP_PKEY* key = EVP_EC_gen("P-256");
  if (!key) {
    if (err) *err = "key generation failed";
    return false;
  }
  X509* x = new_cert(key, "everserve-ca", days, 1);
  X509_set_issuer_name(x, X509_get_subject_name(x));
  add_ext(x, x, NID_basic_constraints, "critical,CA:TRUE");
  add_ext(x, x, NID_key_usage, "critical,keyCertSign,cRLSign");
  const bool ok = X509_sign(x, key, EVP_sha256()) > 0 && write_pem(dir + "/ca.key", key, nullptr) &&
                  write_pem(dir + "/ca.crt", nullptr, x);
  if (!ok && err) *err = "cannot write the CA into " + dir;
  X509_free(x);
  EVP_PKEY_free(key);
  return ok;
}

bool issue(const std::string& dir, const std::string& name, int days, std::string* err) {
  FILE* fk = fopen((dir + "/ca.key").c_str(), "r");
  FILE* fc = fopen((dir + "/ca.crt").c_str(), "r");
  if (!fk || !fc) {
    if (fk) fclose(fk);
    if (fc) fclose(fc);
    if (err) *err = "no CA in " + dir + " (everserve-ctl certs init first)";
    return false;
  }
  EVP_PKEY* ca_key = PEM_read_PrivateKey(fk, nullptr, nullptr, nullptr);
  X509* ca = PEM_read_X509(fc, nullptr, nullptr, nullptr);
  fclose(fk);
  fclose(fc);
  EVP_PKEY* key = EVP_EC_gen("P-256");
  bool ok = ca_key && ca && key;
  if (ok) {
    X509* x = new_cert(key, name, days, (long)(now_us() & 0x7fffffff));
    X509_set_issuer_name(x, X509_get_subject_name(ca));
    const std::string san = "DNS:" + name + ",DNS:localhost,IP:127.0.0.1";
    add_ext(x, ca, NID_subject_alt_name, san.c_str());
    add_ext(x, ca, NID_basic_constraints, "critical,CA:FALSE");
    add_ext(x, ca, NID_ext_key_usage, "serverAuth,clientAuth");
    ok = X509_sign(x, ca_key, EVP_sha256()) > 0 && write_pem(dir + "/" + name + ".key", key, nullptr) &&
         write_pem(dir + "/" + name + ".crt", nullptr, x);
    X509_free(x);
  }
  if (!ok && err) *err = "cannot issue a certificate for " + name;
  EVP_PKEY_free(key);
  EVP_PKEY_free(ca_key);
  X509_free(ca);
  return ok;
}

static std::string pem_of(EVP_PKEY* key, bool private_part) {
  BIO* b = BIO_new(BIO_s_mem());
  const int ok = private_part ? PEM_write_bio_PrivateKey(b, key, nullptr, nullptr, 0, nullptr, nullptr)
                              : PEM_write_bio_PUBKEY(b, key);
  std::string out;
  if (ok == 1) {
    char* p = nullptr;
    const long n = BIO_get_mem_data(b, &p);
    out.assign(p, (size_t)n);
  }
  BIO_free(b);
  return out;
}

bool make_key(std::string& key_pem, std::string& pub_pem, std::string* err) {
  EVP_PKEY* key = EVP_EC_gen("P-256");
  if (!key) {
    if (err) *err = "key generation failed";
    return false;
  }
  key_pem = pem_of(key, true);
  pub_pem = pem_of(key, false);
  EVP_PKEY_free(key);
  return !key_pem.empty() && !pub_pem.empty();
}

bool sign_node(const std::string& ca_dir, const std::string& node, const std::string& pub_pem, int hours,
               std::string& cert_pem, std::string& ca_pem, int64_t& not_after_ms, std::string* err) {
  FILE* fk = fopen((ca_dir + "/ca.key").c_str(), "r");
  FILE* fc = fopen((ca_dir + "/ca.crt").c_str(), "r");
  if (!fk || !fc) {
    if (fk) fclose(fk);
    if (fc) fclose(fc);
    if (err) *err = "this coordinator holds no CA key";
    return false;
  }
  EVP_PKEY* ca_key = PEM_read_PrivateKey(fk, nullptr, nullptr, nullptr);
  X509* ca = PEM_read_X509(fc, nullptr, nullptr, nullptr);
  fclose(fk);
  fclose(fc);
  BIO* b = BIO_new_mem_buf(pub_pem.data(), (int)pub_pem.size());
  EVP_PKEY* pub = PEM_read_bio_PUBKEY(b, nullptr, nullptr, nullptr);
  BIO_free(b);
  bool ok = ca_key && ca && pub;
  if (!pub && err) *err = "the public key does not parse";
  if (ok) {
    X509* x = X509_new();
    X509_set_version(x, 2);
    ASN1_INTEGER_set(X509_get_serialNumber(x), (long)(now_us() & 0x7fffffff));
    X509_gmtime_adj(X509_getm_notBefore(x), -60);
    X509_gmtime_adj(X509_getm_notAfter(x), (long)hours * 3600);
    X509_set_pubkey(x, pub);
    X509_NAME_add_entry_by_txt(X509_get_subject_name(x), "CN", MBSTRING_ASC,
                               reinterpret_cast<const unsigned char*>(node.c_str()), -1, -1, 0);
    X509_set_issuer_name(x, X509_get_subject_name(ca));
    const std::string san = "DNS:" + node;
    add_ext(x, ca, NID_subject_alt_name, san.c_str());
    add_ext(x, ca, NID_basic_constraints, "critical,CA:FALSE");
    add_ext(x, ca, NID_ext_key_usage, "serverAuth,clientAuth");
    ok = X509_sign(x, ca_key, EVP_sha256()) > 0;
    if (ok) {
      BIO* o = BIO_new(BIO_s_mem());
      PEM_write_bio_X509(o, x);
      char* p = nullptr;
      const long n = BIO_get_mem_data(o, &p);
      cert_pem.assign(p, (size_t)n);
      BIO_free(o);
      BIO* c = BIO_new(BIO_s_mem());
      PEM_write_bio_X509(c, ca);
      p = nullptr;
      const long m = BIO_get_mem_data(c, &p);
      ca_pem.assign(p, (size_t)m);
      BIO_free(c);
      not_after_ms = (int64_t)(std::time(nullptr) + (time_t)hours * 3600) * 1000;
    } else if (err) {
      *err = "signing failed";
    }
    X509_free(x);
  }
  EVP_PKEY_free(pub);
  EVP_PKEY_free(ca_key);
  X509_free(ca);
  return ok;
}

}  // namespace tls

std::string sha256_hex(const std::string& data) {
  unsigned char md[EVP_MAX_MD_SIZE];
  unsigned int n = 0;
  EVP_Digest(data.data(), data.size(), md, &n, EVP_sha256(), nullptr);
  static const char* d = "0123456789abcdef";
  std::string out;
  for (unsigned int i = 0; i < n; i++) {
    out.push_back(d[md[i] >> 4]);
    out.push_back(d[md[i] & 15]);
  }
  return out;
}

}  // namespace es
