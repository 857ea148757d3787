// Argument checks of the torch-facing code.
//
// Messages are assembled with std::to_string and string concatenation, and
// TORCH_CHECK only ever receives one finished std::string: with the PyTorch
// build this extension targets, inserting a number into a std::ostream from
// inside a torch extension crashes the process (a three-line extension doing
// `std::ostringstream s; s << 5;` segfaults), so c10::str must not see numbers.
#pragma once

#include <c10/util/Exception.h>

#include <string>
#include <type_traits>

namespace mgfa::detail {

inline void append(std::string& s, const char* v) { s += v; }
inline void append(std::string& s, const std::string& v) { s += v; }
inline void append(std::string& s, char v) { s += v; }
inline void append(std::string& s, bool v) { s += v ? "true" : "false"; }
template <class T>
std::enable_if_t<std::is_arithmetic_v<T>> append(std::string& s, T v) {
  s += std::to_string(v);
}

template <class... A>
std::string msg(const A&... a) {
  std::string s;
  (append(s, a), ...);
  return s;
}

}  // namespace mgfa::detail

// TORCH_CHECK with a message built without streams; at least one message part.
#define MGFA_CHECK(cond, ...) TORCH_CHECK(cond, ::mgfa::detail::msg(__VA_ARGS__))
