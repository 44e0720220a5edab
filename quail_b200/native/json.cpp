#include <cmath>
#include <cstdio>

#include "native.h"

namespace qbn {

std::string json_escape(const std::string& s) {
  std::string o;
  o.reserve(s.size() + 2);
  o += '"';
  for (unsigned char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      default:
        if (c < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof buf, "\\u%04x", c);
          o += buf;
        } else {
          o += (char)c;
        }
    }
  }
  o += '"';
  return o;
}

std::string Json::dump() const {
  switch (kind_) {
    case Kind::Null: return "null";
    case Kind::Bool: return b_ ? "true" : "false";
    case Kind::Int: return std::to_string(i_);
    case Kind::Float: {
      if (!std::isfinite(d_)) return "null";
      char buf[32];
      std::snprintf(buf, sizeof buf, "%.17g", d_);
      std::string s(buf);
      if (s.find_first_of(".eE") == std::string::npos) s += ".0";
      return s;
    }
    case Kind::String: return json_escape(s_);
    case Kind::Array: {
      std::string o = "[";
      for (size_t i = 0; i < arr_.size(); ++i) {
        if (i) o += ",";
        o += arr_[i].dump();
      }
      return o + "]";
    }
    case Kind::Object: {
      std::string o = "{";
      for (size_t i = 0; i < obj_.size(); ++i) {
        if (i) o += ",";
        o += json_escape(obj_[i].first) + ":" + obj_[i].second.dump();
      }
      return o + "}";
    }
  }
  return "null";
}

}  // namespace qbn
