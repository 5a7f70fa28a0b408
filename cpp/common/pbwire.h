// Protobuf binary wire format (proto3): varints, zigzag, fixed32/64, length-delimited fields and
// packed repeated scalars. The generated message structs (everserve_pb.h) call these helpers.
#pragma once

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

namespace pbwire {

enum WireType : uint32_t { kVarint = 0, kI64 = 1, kLen = 2, kI32 = 5 };

inline void varint(std::string& out, uint64_t v) {
  while (v >= 0x80) {
    out.push_back(static_cast<char>((v & 0x7F) | 0x80));
    v >>= 7;
  }
  out.push_back(static_cast<char>(v));
}
inline void key(std::string& out, uint32_t num, WireType wt) { varint(out, (uint64_t(num) << 3) | wt); }

template <class T>
inline void put_varint(std::string& out, uint32_t num, T v) {
  key(out, num, kVarint);
  varint(out, static_cast<uint64_t>(static_cast<int64_t>(v)));  // negative int32 -> 10 bytes
}
inline void put_varint(std::string& out, uint32_t num, bool v) {
  key(out, num, kVarint);
  varint(out, v ? 1 : 0);
}
template <class T>
inline void put_zigzag(std::string& out, uint32_t num, T v) {
  key(out, num, kVarint);
  const int64_t s = static_cast<int64_t>(v);
  varint(out, (static_cast<uint64_t>(s) << 1) ^ static_cast<uint64_t>(s >> 63));
}
template <class T>
inline void put_f32(std::string& out, uint32_t num, T v) {
  key(out, num, kI32);
  uint32_t u;
  if constexpr (std::is_floating_point<T>::value) {
    float f = static_cast<float>(v);
    std::memcpy(&u, &f, 4);
  } else {
    u = static_cast<uint32_t>(v);
  }
  out.append(reinterpret_cast<const char*>(&u), 4);
}
template <class T>
inline void put_f64(std::string& out, uint32_t num, T v) {
  key(out, num, kI64);
  uint64_t u;
  if constexpr (std::is_floating_point<T>::value) {
    double d = static_cast<double>(v);
    std::memcpy(&u, &d, 8);
  } else {
    u = static_cast<uint64_t>(v);
  }
  out.append(reinterpret_cast<const char*>(&u), 8);
}
inline void put_len(std::string& out, uint32_t num, const std::string& s) {
  key(out, num, kLen);
  varint(out, s.size());
  out.append(s);
}
template <class T>
inline void put_packed_varint(std::string& out, uint32_t num, const std::vector<T>& v) {
  if (v.empty()) return;
  std::string body;
  for (const auto& x : v) varint(body, static_cast<uint64_t>(static_cast<int64_t>(x)));
  put_len(out, num, body);
}
inline void put_packed_varint(std::string& out, uint32_t num, const std::vector<bool>& v) {
  if (v.empty()) return;
  std::string body;
  for (bool x : v) varint(body, x ? 1 : 0);
  put_len(out, num, body);
}
template <class T>
inline void put_packed_zigzag(std::string& out, uint32_t num, const std::vector<T>& v) {
  if (v.empty()) return;
  std::string body;
  for (const auto& x : v) {
    const int64_t s = static_cast<int64_t>(x);
    varint(body, (static_cast<uint64_t>(s) << 1) ^ static_cast<uint64_t>(s >> 63));
  }
  put_len(out, num, body);
}
template <class T>
inline void put_packed_f32(std::string& out, uint32_t num, const std::vector<T>& v) {
  if (v.empty()) return;
  std::string body;
  for (const auto& x : v) {
    uint32_t u;
    if constexpr (std::is_floating_point<T>::value) {
      float f = static_cast<float>(x);
      std::memcpy(&u, &f, 4);
    } else {
      u = static_cast<uint32_t>(x);
    }
    body.append(reinterpret_cast<const char*>(&u), 4);
  }
  put_len(out, num, body);
}
template <class T>
inline void put_packed_f64(std::string& out, uint32_t num, const std::vector<T>& v) {
  if (v.empty()) return;
  std::string body;
  for (const auto& x : v) {
    uint64_t u;
    if constexpr (std::is_floating_point<T>::value) {
      double d = static_cast<double>(x);
      std::memcpy(&u, &d, 8);
    } else {
      u = static_cast<uint64_t>(x);
    }
    body.append(reinterpret_cast<const char*>(&u), 8);
  }
  put_len(out, num, body);
}

struct Reader {
  const uint8_t* p;
  const uint8_t* end;
  bool varint(uint64_t& v) {
    v = 0;
    for (int shift = 0; shift < 64; shift += 7) {
      if (p >= end) return false;
      const uint8_t b = *p++;
      v |= uint64_t(b & 0x7F) << shift;
      if (!(b & 0x80)) return true;
    }
    return false;
  }
  bool bytes(const uint8_t*& b, size_t& n) {
    uint64_t len;
    if (!varint(len) || len > size_t(end - p)) return false;
    b = p;
    n = size_t(len);
    p += len;
    return true;
  }
  bool skip(uint32_t wt) {
    uint64_t v;
    switch (wt) {
      case kVarint: return varint(v);
      case kI64: if (end - p < 8) return false; p += 8; return true;
      case kI32: if (end - p < 4) return false; p += 4; return true;
      case kLen: { const uint8_t* b; size_t n; return bytes(b, n); }
      default: return false;
    }
  }
};

template <class T>
inline bool get_varint(Reader& r, uint32_t wt, T& v) {
  uint64_t x;
  if (wt != kVarint || !r.varint(x)) return false;
  v = static_cast<T>(x);
  return true;
}
inline bool get_varint(Reader& r, uint32_t wt, bool& v) {
  uint64_t x;
  if (wt != kVarint || !r.varint(x)) return false;
  v = x != 0;
  return true;
}
template <class T>
inline bool get_zigzag(Reader& r, uint32_t wt, T& v) {
  uint64_t x;
  if (wt != kVarint || !r.varint(x)) return false;
  v = static_cast<T>(static_cast<int64_t>((x >> 1) ^ (~(x & 1) + 1)));
  return true;
}
template <class T>
inline bool get_f32(Reader& r, uint32_t wt, T& v) {
  if (wt != kI32 || r.end - r.p < 4) return false;
  uint32_t u;
  std::memcpy(&u, r.p, 4);
  r.p += 4;
  if constexpr (std::is_floating_point<T>::value) {
    float f;
    std::memcpy(&f, &u, 4);
    v = static_cast<T>(f);
  } else {
    v = static_cast<T>(u);
  }
  return true;
}
template <class T>
inline bool get_f64(Reader& r, uint32_t wt, T& v) {
  if (wt != kI64 || r.end - r.p < 8) return false;
  uint64_t u;
  std::memcpy(&u, r.p, 8);
  r.p += 8;
  if constexpr (std::is_floating_point<T>::value) {
    double d;
    std::memcpy(&d, &u, 8);
    v = static_cast<T>(d);
  } else {
    v = static_cast<T>(u);
  }
  return true;
}
inline bool get_len(Reader& r, uint32_t wt, std::string& s) {
  const uint8_t* b;
  size_t n;
  if (wt != kLen || !r.bytes(b, n)) return false;
  s.assign(reinterpret_cast<const char*>(b), n);
  return true;
}
template <class M>
inline bool get_msg(Reader& r, uint32_t wt, M& m) {
  const uint8_t* b;
  size_t n;
  if (wt != kLen || !r.bytes(b, n)) return false;
  return m.decode(b, n);
}
// repeated scalars arrive packed (proto3 default) or one per key: accept both
template <class T>
inline bool get_repeated_varint(Reader& r, uint32_t wt, std::vector<T>& v) {
  if (wt == kLen) {
    const uint8_t* b;
    size_t n;
    if (!r.bytes(b, n)) return false;
    Reader sub{b, b + n};
    while (sub.p < sub.end) {
      T x;
      if (!get_varint(sub, kVarint, x)) return false;
      v.push_back(x);
    }
    return true;
  }
  T x;
  if (!get_varint(r, wt, x)) return false;
  v.push_back(x);
  return true;
}
inline bool get_repeated_varint(Reader& r, uint32_t wt, std::vector<bool>& v) {
  std::vector<uint64_t> tmp;
  if (!get_repeated_varint(r, wt, tmp)) return false;
  for (auto x : tmp) v.push_back(x != 0);
  return true;
}
template <class T>
inline bool get_repeated_zigzag(Reader& r, uint32_t wt, std::vector<T>& v) {
  if (wt == kLen) {
    const uint8_t* b;
    size_t n;
    if (!r.bytes(b, n)) return false;
    Reader sub{b, b + n};
    while (sub.p < sub.end) {
      T x;
      if (!get_zigzag(sub, kVarint, x)) return false;
      v.push_back(x);
    }
    return true;
  }
  T x;
  if (!get_zigzag(r, wt, x)) return false;
  v.push_back(x);
  return true;
}
template <class T>
inline bool get_repeated_f32(Reader& r, uint32_t wt, std::vector<T>& v) {
  if (wt == kLen) {
    const uint8_t* b;
    size_t n;
    if (!r.bytes(b, n) || n % 4) return false;
    Reader sub{b, b + n};
    while (sub.p < sub.end) {
      T x;
      if (!get_f32(sub, kI32, x)) return false;
      v.push_back(x);
    }
    return true;
  }
  T x;
  if (!get_f32(r, wt, x)) return false;
  v.push_back(x);
  return true;
}
template <class T>
inline bool get_repeated_f64(Reader& r, uint32_t wt, std::vector<T>& v) {
  if (wt == kLen) {
    const uint8_t* b;
    size_t n;
    if (!r.bytes(b, n) || n % 8) return false;
    Reader sub{b, b + n};
    while (sub.p < sub.end) {
      T x;
      if (!get_f64(sub, kI64, x)) return false;
      v.push_back(x);
    }
    return true;
  }
  T x;
  if (!get_f64(r, wt, x)) return false;
  v.push_back(x);
  return true;
}

}  // namespace pbwire
