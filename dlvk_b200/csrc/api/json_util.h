// JSON text helpers of the C++ API (private header).  Numbers are written
// the way Python's json module writes floats (shortest round-trip digits;
// fixed notation for decimal exponents in [-4, 16), else d.ddde+XX), so
// metadata written by either front end is byte-identical.
#pragma once
#include <charconv>
#include <cmath>
#include <cstdio>
#include <string>

namespace dlvk {
namespace json {

inline std::string str(const std::string& s) {
  std::string o = "\"";
  for (char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\t': o += "\\t"; break;
      default:
        if ((unsigned char)c < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof buf, "\\u%04x", c);
          o += buf;
        } else {
          o += c;
        }
    }
  }
  return o + "\"";
}

// Python repr() of a float.
inline std::string num(double v) {
  if (std::isnan(v)) return "NaN";
  if (std::isinf(v)) return v > 0 ? "Infinity" : "-Infinity";
  if (v == 0.0) return std::signbit(v) ? "-0.0" : "0.0";
  char buf[64];
  auto r = std::to_chars(buf, buf + sizeof buf, v, std::chars_format::scientific);
  std::string sci(buf, r.ptr);  // [-]d[.ddd]e[+-]XX, shortest round-trip digits
  const size_t e = sci.find('e');
  const int exp10 = std::stoi(sci.substr(e + 1));
  std::string mant = sci.substr(0, e);
  const bool neg = mant[0] == '-';
  if (neg) mant.erase(0, 1);
  std::string digits;
  for (char c : mant)
    if (c != '.') digits += c;
  std::string out;
  if (exp10 >= -4 && exp10 < 16) {
    if (exp10 < 0) {
      out = "0." + std::string((size_t)(-exp10 - 1), '0') + digits;
    } else if ((int)digits.size() <= exp10 + 1) {
      out = digits + std::string((size_t)(exp10 + 1 - (int)digits.size()), '0') + ".0";
    } else {
      out = digits.substr(0, (size_t)exp10 + 1) + "." + digits.substr((size_t)exp10 + 1);
    }
  } else {
    out = digits.substr(0, 1);
    if (digits.size() > 1) out += "." + digits.substr(1);
    char eb[16];
    std::snprintf(eb, sizeof eb, "e%c%02d", exp10 < 0 ? '-' : '+', std::abs(exp10));
    out += eb;
  }
  return neg ? "-" + out : out;
}

}  // namespace json
}  // namespace dlvk
