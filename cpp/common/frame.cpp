#include "frame.h"

#include <errno.h>
#include <poll.h>
#include <unistd.h>

#include <cstring>

namespace es {

bool encode_frame(const std::string& payload, std::string& out) {
  if (payload.size() > kMaxFrame) return false;
  const uint32_t n = static_cast<uint32_t>(payload.size());
  const char hdr[4] = {static_cast<char>(n >> 24), static_cast<char>(n >> 16), static_cast<char>(n >> 8),
                       static_cast<char>(n)};
  out.append(hdr, 4);
  out.append(payload);
  return true;
}

bool FrameReader::feed(const char* data, size_t n) {
  if (pos_ > 0 && pos_ >= buf_.size() / 2) {  // compact
    buf_.erase(0, pos_);
    pos_ = 0;
  }
  buf_.append(data, n);
  if (buffered() >= 4) {
    const auto* p = reinterpret_cast<const uint8_t*>(buf_.data() + pos_);
    const uint32_t len = (uint32_t(p[0]) << 24) | (uint32_t(p[1]) << 16) | (uint32_t(p[2]) << 8) | p[3];
    if (len > kMaxFrame) return false;
  }
  return true;
}

bool FrameReader::next(std::string& out) {
  if (buffered() < 4) return false;
  const auto* p = reinterpret_cast<const uint8_t*>(buf_.data() + pos_);
  const uint32_t len = (uint32_t(p[0]) << 24) | (uint32_t(p[1]) << 16) | (uint32_t(p[2]) << 8) | p[3];
  if (buffered() < 4 + size_t(len)) return false;
  out.assign(buf_.data() + pos_ + 4, len);
  pos_ += 4 + len;
  if (pos_ == buf_.size()) {
    buf_.clear();
    pos_ = 0;
  }
  return true;
}

static bool write_all(int fd, const char* p, size_t n) {
  while (n > 0) {
    const ssize_t w = ::write(fd, p, n);
    if (w < 0) {
      if (errno == EINTR) continue;
      if (errno == EAGAIN) {
        pollfd pf{fd, POLLOUT, 0};
        ::poll(&pf, 1, 1000);
        continue;
      }
      return false;
    }
    p += w;
    n -= size_t(w);
  }
  return true;
}

bool write_frame(int fd, const std::string& payload) {
  std::string out;
  if (!encode_frame(payload, out)) return false;
  return write_all(fd, out.data(), out.size());
}

static bool read_exact(int fd, char* p, size_t n, int timeout_ms) {
  while (n > 0) {
    if (timeout_ms >= 0) {
      pollfd pf{fd, POLLIN, 0};
      const int r = ::poll(&pf, 1, timeout_ms);
      if (r <= 0) return false;
    }
    const ssize_t got = ::read(fd, p, n);
    if (got < 0 && errno == EINTR) continue;
    if (got <= 0) return false;
    p += got;
    n -= size_t(got);
  }
  return true;
}

bool read_frame(int fd, std::string& payload, int timeout_ms) {
  char hdr[4];
  if (!read_exact(fd, hdr, 4, timeout_ms)) return false;
  const auto* p = reinterpret_cast<const uint8_t*>(hdr);
  const uint32_t len = (uint32_t(p[0]) << 24) | (uint32_t(p[1]) << 16) | (uint32_t(p[2]) << 8) | p[3];
  if (len > kMaxFrame) return false;
  payload.resize(len);
  return read_exact(fd, payload.data(), len, timeout_ms);
}

}  // namespace es
