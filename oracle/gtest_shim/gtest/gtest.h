// Minimal GoogleTest-compatible harness (own implementation, test
// infrastructure only).  It provides the subset of the gtest API that the
// reference's tests/test_cuda.cpp uses -- TEST, GTEST_SKIP, the EXPECT_* /
// ASSERT_* comparison macros with `<<` messages, EXPECT_THROW /
// EXPECT_NO_THROW -- so that file compiles unchanged (googletest itself is
// not available offline).  Link gtest_shim_main.cpp for main().
#pragma once

#include <cmath>
#include <cstring>
#include <functional>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

namespace gtest_shim {

struct TestCase {
  const char* suite;
  const char* name;
  void (*fn)();
};

inline std::vector<TestCase>& registry() {
  static std::vector<TestCase> r;
  return r;
}

struct State {
  bool failed = false;
  bool skipped = false;
  long failures = 0;
};
inline State& state() {
  static State s;
  return s;
}

struct Registrar {
  Registrar(const char* suite, const char* name, void (*fn)()) {
    registry().push_back({suite, name, fn});
  }
};

class Message {
 public:
  template <class T>
  Message& operator<<(const T& v) {
    os_ << v;
    return *this;
  }
  std::string str() const { return os_.str(); }

 private:
  std::ostringstream os_;
};

class FailureHelper {
 public:
  FailureHelper(const char* file, int line, std::string what)
      : file_(file), line_(line), what_(std::move(what)) {}
  void operator=(const Message& m) const {
    State& s = state();
    s.failed = true;
    if (++s.failures <= 50) {
      std::cerr << file_ << ":" << line_ << ": Failure: " << what_;
      const std::string extra = m.str();
      if (!extra.empty()) std::cerr << " | " << extra;
      std::cerr << "\n";
    }
  }

 private:
  const char* file_;
  int line_;
  std::string what_;
};

class SkipHelper {
 public:
  void operator=(const Message&) const { state().skipped = true; }
};

template <class A, class B>
std::string describe(const char* op, const char* ea, const char* eb, const A& a,
                     const B& b) {
  std::ostringstream os;
  os << ea << " " << op << " " << eb << " (" << a << " vs " << b << ")";
  return os.str();
}

inline bool float_eq(float a, float b) {
  if (a == b) return true;
  const float diff = std::fabs(a - b);
  const float scale = std::fmax(std::fabs(a), std::fabs(b));
  return diff <= scale * 4 * 1.1920929e-7f;
}

}  // namespace gtest_shim

#define TEST(suite, name)                                                   \
  static void suite##_##name##_body();                                      \
  static ::gtest_shim::Registrar suite##_##name##_registrar(                \
      #suite, #name, &suite##_##name##_body);                               \
  static void suite##_##name##_body()

#define GTEST_SKIP() return ::gtest_shim::SkipHelper() = ::gtest_shim::Message()

#define GTEST_SHIM_CHECK_(cond, text, on_fail)                               \
  if (cond)                                                                  \
    ;                                                                        \
  else                                                                       \
    on_fail ::gtest_shim::FailureHelper(__FILE__, __LINE__, text) =          \
        ::gtest_shim::Message()

#define GTEST_SHIM_CMP_(a, b, op, on_fail)                                   \
  GTEST_SHIM_CHECK_((a)op(b),                                                \
                    ::gtest_shim::describe(#op, #a, #b, (a), (b)), on_fail)

#define EXPECT_EQ(a, b) GTEST_SHIM_CMP_(a, b, ==, )
#define EXPECT_NE(a, b) GTEST_SHIM_CMP_(a, b, !=, )
#define EXPECT_LT(a, b) GTEST_SHIM_CMP_(a, b, <, )
#define EXPECT_LE(a, b) GTEST_SHIM_CMP_(a, b, <=, )
#define EXPECT_GT(a, b) GTEST_SHIM_CMP_(a, b, >, )
#define EXPECT_GE(a, b) GTEST_SHIM_CMP_(a, b, >=, )
#define ASSERT_EQ(a, b) GTEST_SHIM_CMP_(a, b, ==, return)
#define ASSERT_NE(a, b) GTEST_SHIM_CMP_(a, b, !=, return)
#define EXPECT_TRUE(c) GTEST_SHIM_CHECK_(static_cast<bool>(c), #c, )
#define EXPECT_FALSE(c) GTEST_SHIM_CHECK_(!static_cast<bool>(c), "!" #c, )
#define ASSERT_TRUE(c) GTEST_SHIM_CHECK_(static_cast<bool>(c), #c, return)
#define EXPECT_NEAR(a, b, tol)                                               \
  GTEST_SHIM_CHECK_(std::fabs(double(a) - double(b)) <= double(tol),         \
                    ::gtest_shim::describe("~=", #a, #b, (a), (b)), )
#define EXPECT_FLOAT_EQ(a, b)                                                \
  GTEST_SHIM_CHECK_(::gtest_shim::float_eq((a), (b)),                        \
                    ::gtest_shim::describe("==f", #a, #b, (a), (b)), )
#define EXPECT_STREQ(a, b)                                                   \
  GTEST_SHIM_CHECK_(std::strcmp((a), (b)) == 0,                              \
                    ::gtest_shim::describe("streq", #a, #b, (a), (b)), )

#define EXPECT_THROW(stmt, exc)                                              \
  do {                                                                       \
    bool gtest_shim_caught_ = false;                                         \
    try {                                                                    \
      stmt;                                                                  \
    } catch (const exc&) {                                                   \
      gtest_shim_caught_ = true;                                             \
    } catch (...) {                                                          \
    }                                                                        \
    if (!gtest_shim_caught_)                                                 \
      ::gtest_shim::FailureHelper(__FILE__, __LINE__,                        \
                                  "expected " #exc " from " #stmt) =         \
          ::gtest_shim::Message();                                           \
  } while (false)

#define EXPECT_NO_THROW(stmt)                                                \
  do {                                                                       \
    try {                                                                    \
      stmt;                                                                  \
    } catch (...) {                                                          \
      ::gtest_shim::FailureHelper(__FILE__, __LINE__,                        \
                                  "unexpected exception from " #stmt) =      \
          ::gtest_shim::Message();                                           \
    }                                                                        \
  } while (false)
