// Argument checks of the Python bindings. A failed check throws std::runtime_error (pybind11 turns it
// into RuntimeError) from one out-of-line function; messages are assembled with std::string.
#pragma once

#include <string>
#include <type_traits>

namespace cob {

[[noreturn]] void fail(const std::string& msg);

inline std::string piece(const std::string& s) { return s; }
inline std::string piece(const char* s) { return s ? std::string(s) : std::string("(null)"); }
template <typename T, typename std::enable_if<std::is_arithmetic<T>::value, int>::type = 0>
std::string piece(T v) {
  return std::to_string(v);
}
inline std::string msg() { return std::string(); }
template <typename A, typename... R>
std::string msg(const A& a, const R&... r) {
  return piece(a) + msg(r...);
}

}  // namespace cob

#define COB_CHECK(cond, ...)                    \
  do {                                          \
    if (!(cond)) ::cob::fail(::cob::msg(__VA_ARGS__)); \
  } while (0)
