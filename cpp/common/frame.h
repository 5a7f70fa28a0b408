// Length-prefixed frames: a 4-byte big-endian payload length, then the payload (one protobuf
// message). Frames above kMaxFrame are refused by both writer and reader. FrameReader accumulates
// bytes from non-blocking reads and yields complete frames, so a frame split across reads (or
// several frames in one read) is handled.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace es {

constexpr size_t kMaxFrame = 16u << 20;

// Append one frame to `out`; false if the payload is too large.
bool encode_frame(const std::string& payload, std::string& out);

class FrameReader {
 public:
  // Feed bytes; false on a malformed stream (a length above kMaxFrame).
  bool feed(const char* data, size_t n);
  // Pop the next complete frame into `out`; false when none is complete yet.
  bool next(std::string& out);
  size_t buffered() const { return buf_.size() - pos_; }

 private:
  std::string buf_;
  size_t pos_ = 0;
};

// Blocking helpers for simple clients: write a whole frame / read one frame (timeout_ms < 0: none).
bool write_frame(int fd, const std::string& payload);
bool read_frame(int fd, std::string& payload, int timeout_ms = -1);

}  // namespace es
