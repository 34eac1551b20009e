// check.hpp -- minimal self-registering test harness for the C++ host-API tests.
//
//   TEST(name) { CHECK(cond); CHECK_EQ(a, b); CHECK_THROWS_WITH(expr, "substring"); }
//
// main() runs every registered test (or those whose name contains argv[1]), prints one
// line per test and exits non-zero if any check failed.
#pragma once

#include <cmath>
#include <cstdio>
#include <cstring>
#include <exception>
#include <functional>
#include <sstream>
#include <string>
#include <vector>

namespace check {

struct Case {
  const char* name;
  std::function<void()> fn;
};

inline std::vector<Case>& registry() {
  static std::vector<Case> r;
  return r;
}

struct Failure {
  std::string what;
};

struct Register {
  Register(const char* name, std::function<void()> fn) { registry().push_back({name, std::move(fn)}); }
};

template <typename T>
std::string show(const T& v) {
  std::ostringstream os;
  os << v;
  return os.str();
}
template <typename T>
std::string show(const std::vector<T>& v) {
  std::ostringstream os;
  os << "[";
  for (size_t i = 0; i < v.size(); ++i) os << (i ? ", " : "") << v[i];
  os << "]";
  return os.str();
}

inline void fail(const char* file, int line, const std::string& msg) {
  throw Failure{std::string(file) + ":" + std::to_string(line) + ": " + msg};
}

inline int run_all(int argc, char** argv) {
  const char* filter = argc > 1 ? argv[1] : nullptr;
  int failed = 0, ran = 0;
  for (const Case& c : registry()) {
    if (filter && !std::strstr(c.name, filter)) continue;
    ++ran;
    try {
      c.fn();
      std::printf("PASS %s\n", c.name);
    } catch (const Failure& f) {
      ++failed;
      std::printf("FAIL %s: %s\n", c.name, f.what.c_str());
    } catch (const std::exception& e) {
      ++failed;
      std::printf("FAIL %s: unexpected exception: %s\n", c.name, e.what());
    }
  }
  std::printf("%d passed, %d failed\n", ran - failed, failed);
  return failed ? 1 : 0;
}

}  // namespace check

#define CHECK_CAT2(a, b) a##b
#define CHECK_CAT(a, b) CHECK_CAT2(a, b)
#define TEST(name)                                                         \
  static void name();                                                      \
  static ::check::Register CHECK_CAT(reg_, name)(#name, name);             \
  static void name()

#define CHECK(cond)                                                        \
  do {                                                                     \
    if (!(cond)) ::check::fail(__FILE__, __LINE__, "CHECK(" #cond ")");    \
  } while (0)

#define CHECK_EQ(a, b)                                                                           \
  do {                                                                                           \
    const auto va_ = (a);                                                                        \
    const auto vb_ = (b);                                                                        \
    if (!(va_ == vb_))                                                                           \
      ::check::fail(__FILE__, __LINE__,                                                          \
                    std::string(#a " == " #b ": ") + ::check::show(va_) + " vs " + ::check::show(vb_)); \
  } while (0)

#define CHECK_THROWS_WITH(expr, substr)                                                          \
  do {                                                                                           \
    bool thrown_ = false;                                                                        \
    try {                                                                                        \
      (void)(expr);                                                                              \
    } catch (const std::exception& e_) {                                                         \
      thrown_ = true;                                                                            \
      if (!std::strstr(e_.what(), substr))                                                       \
        ::check::fail(__FILE__, __LINE__, std::string("message '") + e_.what() +                 \
                                              "' lacks '" + (substr) + "'");                     \
    }                                                                                            \
    if (!thrown_) ::check::fail(__FILE__, __LINE__, "no exception from " #expr);                 \
  } while (0)

#define TEST_MAIN() \
  int main(int argc, char** argv) { return ::check::run_all(argc, argv); }
