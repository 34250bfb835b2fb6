// underhfs_cpp_serve: JSON-lines request loop over stdin/stdout.
//
// Protocol (reference cpp/serve_main.cpp): one JSON object per line with an
// "op" member.  {"op":"health"} -> {"status":"ok"}; {"op":"predict",
// "payload":V} -> {"result":V} (V echoed verbatim); {"op":"exit"} or
// {"op":"quit"} ends the loop; anything else -> {"error":"unsupported op"}.
// Unlike the reference's substring search, members are located by a small
// tokenizer that skips strings, nested objects and arrays, so a payload that
// contains the text "op" is not mistaken for the op member.
#include <cctype>
#include <iostream>
#include <string>

namespace {

// Index one past the JSON value starting at s[i] (string, object, array or scalar).
size_t skip_value(const std::string& s, size_t i) {
  if (i >= s.size()) return i;
  const char c = s[i];
  if (c == '"') {
    ++i;
    while (i < s.size() && s[i] != '"') i += (s[i] == '\\') ? 2 : 1;
    return i < s.size() ? i + 1 : i;
  }
  if (c == '{' || c == '[') {
    int depth = 0;
    while (i < s.size()) {
      const char d = s[i];
      if (d == '"') {
        i = skip_value(s, i);
        continue;
      }
      if (d == '{' || d == '[') ++depth;
      if (d == '}' || d == ']') {
        --depth;
        if (depth == 0) return i + 1;
      }
      ++i;
    }
    return i;
  }
  while (i < s.size() && s[i] != ',' && s[i] != '}' && s[i] != ']' && !std::isspace((unsigned char)s[i])) ++i;
  return i;
}

size_t skip_ws(const std::string& s, size_t i) {
  while (i < s.size() && std::isspace((unsigned char)s[i])) ++i;
  return i;
}

// Raw text of the top-level member `key` of the object in `s`, or "" if absent.
std::string member(const std::string& s, const std::string& key) {
  size_t i = skip_ws(s, 0);
  if (i >= s.size() || s[i] != '{') return "";
  ++i;
  while (i < s.size()) {
    i = skip_ws(s, i);
    if (i < s.size() && s[i] == '}') return "";
    if (i >= s.size() || s[i] != '"') return "";
    const size_t kend = skip_value(s, i);
    const std::string k = s.substr(i + 1, kend - i - 2);
    i = skip_ws(s, kend);
    if (i >= s.size() || s[i] != ':') return "";
    i = skip_ws(s, i + 1);
    const size_t vend = skip_value(s, i);
    if (k == key) return s.substr(i, vend - i);
    i = skip_ws(s, vend);
    if (i < s.size() && s[i] == ',') ++i;
  }
  return "";
}

}  // namespace

int main() {
  std::ios::sync_with_stdio(false);
  std::string line;
  while (std::getline(std::cin, line)) {
    const std::string op = member(line, "op");
    if (op == "\"exit\"" || op == "\"quit\"") break;
    if (op == "\"health\"") {
      std::cout << "{\"status\":\"ok\"}" << std::endl;
    } else if (op == "\"predict\"") {
      std::string payload = member(line, "payload");
      if (payload.empty()) payload = "null";
      std::cout << "{\"result\":" << payload << "}" << std::endl;
    } else {
      std::cout << "{\"error\":\"unsupported op\"}" << std::endl;
    }
  }
  return 0;
}
