#include "net.h"
#include "tls.h"

#include <arpa/inet.h>
#include <errno.h>
#include <fcntl.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/eventfd.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstring>

namespace es {

uint64_t now_ms() {
  return (uint64_t)std::chrono::duration_cast<std::chrono::milliseconds>(
             std::chrono::system_clock::now().time_since_epoch())
      .count();
}
uint64_t now_us() {
  return (uint64_t)std::chrono::duration_cast<std::chrono::microseconds>(
             std::chrono::system_clock::now().time_since_epoch())
      .count();
}

bool Address::parse(const std::string& s, Address& out) {
  out = Address{};
  if (s.rfind("unix:", 0) == 0) {
    out.unix_socket = true;
    out.path = s.substr(5);
    return !out.path.empty();
  }
  if (!s.empty() && s[0] == '/') {
    out.unix_socket = true;
    out.path = s;
    return true;
  }
  const auto colon = s.rfind(':');
  if (colon == std::string::npos) return false;
  out.host = s.substr(0, colon);
  if (out.host.size() >= 2 && out.host.front() == '[' && out.host.back() == ']')
    out.host = out.host.substr(1, out.host.size() - 2);
  out.port = atoi(s.substr(colon + 1).c_str());
  return out.port >= 0 && out.port < 65536;
}

std::string Address::str() const { return unix_socket ? "unix:" + path : host + ":" + std::to_string(port); }

static void set_nonblock(int fd) { fcntl(fd, F_SETFL, fcntl(fd, F_GETFL) | O_NONBLOCK); }

int listen_on(const Address& a, std::string* err) {
  int fd = -1;
  if (a.unix_socket) {
    fd = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    sockaddr_un sa{};
    sa.sun_family = AF_UNIX;
    if (a.path.size() >= sizeof(sa.sun_path)) {
      if (err) *err = "socket path too long";
      ::close(fd);
      return -1;
    }
    std::strcpy(sa.sun_path, a.path.c_str());
    ::unlink(a.path.c_str());
    if (::bind(fd, (sockaddr*)&sa, sizeof(sa)) != 0 || ::listen(fd, SOMAXCONN > 4096 ? SOMAXCONN : 4096) != 0) {
      if (err) *err = std::string("bind/listen ") + a.path + ": " + strerror(errno);
      ::close(fd);
      return -1;
    }
  } else {
    fd = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
    int one = 1;
    setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in sa{};
    sa.sin_family = AF_INET;
    sa.sin_port = htons((uint16_t)a.port);
    if (a.host.empty() || a.host == "0.0.0.0") sa.sin_addr.s_addr = INADDR_ANY;
    else inet_pton(AF_INET, a.host == "localhost" ? "127.0.0.1" : a.host.c_str(), &sa.sin_addr);
    if (::bind(fd, (sockaddr*)&sa, sizeof(sa)) != 0 || ::listen(fd, SOMAXCONN > 4096 ? SOMAXCONN : 4096) != 0) {
      if (err) *err = std::string("bind/listen ") + a.str() + ": " + strerror(errno);
      ::close(fd);
      return -1;
    }
  }
  set_nonblock(fd);
  return fd;
}

int connect_to(const Address& a, int timeout_ms, std::string* err) {
  int fd;
  int rc;
  if (a.unix_socket) {
    fd = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    sockaddr_un sa{};
    sa.sun_family = AF_UNIX;
    std::strncpy(sa.sun_path, a.path.c_str(), sizeof(sa.sun_path) - 1);
    set_nonblock(fd);
    rc = ::connect(fd, (sockaddr*)&sa, sizeof(sa));
  } else {
    fd = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
    int one = 1;
    setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
    sockaddr_in sa{};
    sa.sin_family = AF_INET;
    sa.sin_port = htons((uint16_t)a.port);
    if (inet_pton(AF_INET, a.host == "localhost" ? "127.0.0.1" : a.host.c_str(), &sa.sin_addr) != 1) {
      addrinfo hints{}, *res = nullptr;
      hints.ai_family = AF_INET;
      if (getaddrinfo(a.host.c_str(), nullptr, &hints, &res) != 0 || res == nullptr) {
        if (err) *err = "cannot resolve " + a.host;
        ::close(fd);
        return -1;
      }
      sa.sin_addr = reinterpret_cast<sockaddr_in*>(res->ai_addr)->sin_addr;
      freeaddrinfo(res);
    }
    set_nonblock(fd);
    rc = ::connect(fd, (sockaddr*)&sa, sizeof(sa));
  }
  if (rc != 0 && errno != EINPROGRESS && errno != EAGAIN) {
    if (err) *err = std::string("connect ") + a.str() + ": " + strerror(errno);
    ::close(fd);
    return -1;
  }
  if (rc != 0) {
    pollfd pf{fd, POLLOUT, 0};
    if (::poll(&pf, 1, timeout_ms) <= 0) {
      if (err) *err = "connect timeout " + a.str();
      ::close(fd);
      return -1;
    }
    int soerr = 0;
    socklen_t len = sizeof(soerr);
    getsockopt(fd, SOL_SOCKET, SO_ERROR, &soerr, &len);
    if (soerr != 0) {
      if (err) *err = std::string("connect ") + a.str() + ": " + strerror(soerr);
      ::close(fd);
      return -1;
    }
  }
  return fd;
}

bool Loop::listen(const Address& a, AcceptFn on_accept, std::string* err) {
  const int fd = listen_on(a, err);
  if (fd < 0) return false;
  listeners_.push_back({fd, std::move(on_accept), !a.unix_socket});
  return true;
}

Conn* Loop::adopt(int fd, const std::string& peer) {
  set_nonblock(fd);
  auto c = std::make_unique<Conn>();
  c->id = next_id_++;
  c->fd = fd;
  c->peer = peer;
  sockaddr_storage ss{};
  socklen_t sl = sizeof(ss);
  if (tls::enabled() && getsockname(fd, (sockaddr*)&ss, &sl) == 0 && ss.ss_family == AF_INET) {
    c->ssl = tls::new_client(fd);  // an outgoing TCP link: it speaks first
    c->handshaking = true;
    c->hs_want_write = true;
  }
  Conn* raw = c.get();
  conns_[raw->id] = std::move(c);
  return raw;
}

void Loop::progress_handshake(Conn& c) {
  bool ww = false;
  const int r = tls::handshake(c.ssl, &ww);
  if (r == 1) {
    c.handshaking = false;
    c.peer_cn = tls::peer_name(c.ssl);
    flush_conn(c);
    read_conn(c);  // data that came with the last handshake message is already in the session
  } else if (r == 0) {
    c.hs_want_write = ww;
  } else {
    c.closing = true;
    c.out.clear();
  }
}

Conn* Loop::conn(uint64_t id) {
  auto it = conns_.find(id);
  return it == conns_.end() ? nullptr : it->second.get();
}

bool Loop::send(uint64_t id, const std::string& payload) {
  Conn* c = conn(id);
  if (c == nullptr || c->closing) return false;
  if (!encode_frame(payload, c->out)) return false;
  flush_conn(*c);
  return true;
}

void Loop::close(uint64_t id) {
  Conn* c = conn(id);
  if (c != nullptr) c->closing = true;
}

uint64_t Loop::every(uint64_t ms, std::function<void()> fn, bool repeat) {
  const uint64_t id = next_id_++;
  timers_.push_back({id, now_ms() + ms, ms, repeat, std::move(fn)});
  return id;
}

void Loop::cancel(uint64_t timer) {
  timers_.erase(std::remove_if(timers_.begin(), timers_.end(), [&](const Timer& t) { return t.id == timer; }),
                timers_.end());
}

void Loop::watch(int fd, std::function<void()> on_readable) { watched_[fd] = std::move(on_readable); }

Loop::Loop() {
  wake_fd_ = ::eventfd(0, EFD_NONBLOCK | EFD_CLOEXEC);
  if (wake_fd_ >= 0)
    watch(wake_fd_, [this] {
      uint64_t n;
      while (::read(wake_fd_, &n, sizeof n) > 0) {
      }
      std::vector<std::function<void()>> tasks;
      {
        std::lock_guard<std::mutex> g(post_mu_);
        tasks.swap(posted_);
      }
      for (auto& t : tasks) t();
    });
}

Loop::~Loop() {
  if (wake_fd_ >= 0) ::close(wake_fd_);
}

void Loop::post(std::function<void()> fn) {
  {
    std::lock_guard<std::mutex> g(post_mu_);
    posted_.push_back(std::move(fn));
  }
  const uint64_t one = 1;
  if (wake_fd_ >= 0) (void)!::write(wake_fd_, &one, sizeof one);
}

void Loop::flush_conn(Conn& c) {
  if (c.ssl) {
    if (c.handshaking) return;  // queued until the session is up
    while (!c.out.empty()) {
      const long w = tls::write(c.ssl, c.out.data(), c.out.size());
      if (w == -1) return;
      if (w < 0) {
        c.closing = true;
        c.out.clear();
        return;
      }
      c.out.erase(0, size_t(w));
    }
    return;
  }
  while (!c.out.empty()) {
    const ssize_t w = ::send(c.fd, c.out.data(), c.out.size(), MSG_NOSIGNAL);
    if (w < 0) {
      if (errno == EAGAIN || errno == EINTR) return;
      c.closing = true;
      c.out.clear();
      return;
    }
    c.out.erase(0, size_t(w));
  }
}

void Loop::read_conn(Conn& c) {
  char buf[65536];
  if (c.ssl && c.handshaking) {
    progress_handshake(c);
    return;
  }
  while (true) {
    ssize_t n;
    if (c.ssl) {
      const long r = tls::read(c.ssl, buf, sizeof(buf));
      if (r == -1) break;
      n = r == -2 ? -1 : r;
      if (n < 0) {
        c.closing = true;
        break;
      }
    } else {
      n = ::recv(c.fd, buf, sizeof(buf), 0);
    }
    if (n < 0) {
      if (errno == EAGAIN || errno == EINTR) break;
      c.closing = true;
      break;
    }
    if (n == 0) {
      c.closing = true;
      break;
    }
    if (!c.reader.feed(buf, size_t(n))) {
      c.closing = true;
      break;
    }
  }
  std::string frame;
  const uint64_t id = c.id;
  while (c.reader.next(frame)) {
    if (c.on_frame) c.on_frame(c, frame);
    if (conn(id) == nullptr) return;
  }
}

void Loop::drop(uint64_t id) {
  auto it = conns_.find(id);
  if (it == conns_.end()) return;
  std::unique_ptr<Conn> c = std::move(it->second);
  conns_.erase(it);
  if (c->on_close) c->on_close(*c);
  tls::free_session(c->ssl);
  ::close(c->fd);
}

void Loop::run() {
  std::vector<pollfd> pfds;
  while (running_) {
    pfds.clear();
    for (auto& l : listeners_) pfds.push_back({l.fd, POLLIN, 0});
    for (auto& w : watched_) pfds.push_back({w.first, POLLIN, 0});
    std::vector<uint64_t> ids;
    for (auto& kv : conns_) {
      short ev = POLLIN;
      if (kv.second->handshaking) ev = kv.second->hs_want_write ? POLLOUT : POLLIN;
      else if (!kv.second->out.empty()) ev |= POLLOUT;
      pfds.push_back({kv.second->fd, ev, 0});
      ids.push_back(kv.first);
    }
    int timeout = 200;
    const uint64_t now = now_ms();
    for (auto& t : timers_) timeout = std::min<int>(timeout, t.due > now ? int(t.due - now) : 0);
    ::poll(pfds.data(), pfds.size(), timeout);
    size_t i = 0;
    for (; i < listeners_.size(); i++) {
      if (pfds[i].revents & POLLIN) {
        while (true) {
          const int fd = ::accept4(listeners_[i].fd, nullptr, nullptr, SOCK_CLOEXEC);
          if (fd < 0) break;
          Conn* c = adopt(fd, "accepted");
          if (c->ssl) {  // adopt took an accepted socket for an outgoing one
            tls::free_session(c->ssl);
            c->ssl = nullptr;
            c->handshaking = false;
          }
          if (listeners_[i].tcp && tls::enabled()) {
            c->ssl = tls::new_server(fd);
            c->handshaking = true;
            c->hs_want_write = false;
          }
          listeners_[i].on_accept(*c);
        }
      }
    }
    size_t w0 = i;
    {
      std::vector<std::pair<int, std::function<void()>>> ready;
      size_t k = 0;
      for (auto& w : watched_) {
        if (pfds[w0 + k].revents & POLLIN) ready.push_back(w);
        k++;
      }
      i = w0 + watched_.size();
      for (auto& r : ready) r.second();
    }
    for (size_t j = 0; j < ids.size(); j++) {
      Conn* c = conn(ids[j]);
      if (c == nullptr) continue;
      const short re = pfds[i + j].revents;
      if (c->handshaking) {
        if (re & (POLLIN | POLLOUT | POLLHUP | POLLERR)) progress_handshake(*c);
        continue;
      }
      if (re & (POLLIN | POLLHUP | POLLERR)) read_conn(*c);
      c = conn(ids[j]);
      if (c != nullptr && (re & POLLOUT)) flush_conn(*c);
    }
    // timers: one-shot timers leave the list before they run
    const uint64_t t_now = now_ms();
    std::vector<std::function<void()>> due;
    for (auto it = timers_.begin(); it != timers_.end();) {
      if (it->due <= t_now) {
        due.push_back(it->fn);
        if (it->repeat) {
          it->due = t_now + it->period;
          ++it;
        } else {
          it = timers_.erase(it);
        }
      } else {
        ++it;
      }
    }
    for (auto& f : due) f();
    std::vector<uint64_t> dead;
    for (auto& kv : conns_)
      if (kv.second->closing && kv.second->out.empty()) dead.push_back(kv.first);
    for (auto id : dead) drop(id);
  }
}

}  // namespace es
