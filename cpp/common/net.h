// Sockets and a single-threaded poll loop for the control-plane processes.
//
// Addresses are "unix:/path/to.sock" or "host:port" (TCP, TCP_NODELAY). A Loop owns listening
// sockets and connections; each connection reads frames (frame.h) and hands them to a handler on
// the loop thread; writes are queued and flushed when the socket is writable. Timers run on the
// same thread, so handlers never race each other.
#pragma once

#include <cstdint>
#include <functional>
#include <mutex>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "frame.h"

namespace es {

struct Address {
  bool unix_socket = false;
  std::string path;  // unix
  std::string host;  // tcp
  int port = 0;
  static bool parse(const std::string& s, Address& out);
  std::string str() const;
};

int listen_on(const Address& a, std::string* err = nullptr);
int connect_to(const Address& a, int timeout_ms, std::string* err = nullptr);
uint64_t now_ms();
uint64_t now_us();

class Loop;

struct Conn {
  uint64_t id = 0;
  int fd = -1;
  std::string peer;
  FrameReader reader;
  std::string out;
  bool closing = false;
  std::function<void(Conn&, const std::string&)> on_frame;
  std::function<void(Conn&)> on_close;
  void* user = nullptr;  // handler state (owned by the handler)
  // TCP links when TLS is configured (tls.h): the session, its handshake state, and the peer's
  // certificate name once the handshake is done
  void* ssl = nullptr;
  bool handshaking = false;
  bool hs_want_write = false;
  std::string peer_cn;
};

class Loop {
 public:
  using AcceptFn = std::function<void(Conn&)>;
  Loop();
  ~Loop();
  Loop(const Loop&) = delete;
  Loop& operator=(const Loop&) = delete;
  // Listen on `a`; each accepted connection is passed to `on_accept` to install its handlers.
  bool listen(const Address& a, AcceptFn on_accept, std::string* err = nullptr);
  // Adopt a connected socket (an outgoing link).
  Conn* adopt(int fd, const std::string& peer);
  // Queue a frame on a connection (dropped if the connection is gone).
  bool send(uint64_t conn_id, const std::string& payload);
  Conn* conn(uint64_t id);
  void close(uint64_t id);
  // A timer: `fn` runs after `ms`, and again every `ms` if `repeat`.
  uint64_t every(uint64_t ms, std::function<void()> fn, bool repeat = true);
  void cancel(uint64_t timer);
  // A raw readable fd (e.g. an HTTP listener with its own protocol).
  void watch(int fd, std::function<void()> on_readable);
  void run();
  void stop() { running_ = false; }
  // Run `fn` on the loop's thread (the one call that other threads may make).
  void post(std::function<void()> fn);

 private:
  struct Listener {
    int fd;
    AcceptFn on_accept;
    bool tcp;
  };
  void progress_handshake(Conn& c);
  struct Timer {
    uint64_t id, due, period;
    bool repeat;
    std::function<void()> fn;
  };
  void read_conn(Conn& c);
  void flush_conn(Conn& c);
  void drop(uint64_t id);
  std::vector<Listener> listeners_;
  std::map<uint64_t, std::unique_ptr<Conn>> conns_;
  std::vector<Timer> timers_;
  std::map<int, std::function<void()>> watched_;
  uint64_t next_id_ = 1;
  bool running_ = true;
  int wake_fd_ = -1;  // eventfd: a posted task is waiting
  std::mutex post_mu_;
  std::vector<std::function<void()>> posted_;
};

}  // namespace es
