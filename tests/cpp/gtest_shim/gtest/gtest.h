// gtest.h -- TEST INFRASTRUCTURE: a minimal stand-in for the GoogleTest API
// the reference's unit tests use (TEST, EXPECT_* / ASSERT_* with streamed
// messages, testing::InitGoogleTest, RUN_ALL_TESTS), so those test files can
// be compiled unmodified against this repository's frontend and run on the
// GPU box, where GoogleTest is not installed.  Written for this repository;
// it implements only what those files call.
//
// Semantics kept: a failed EXPECT_* records a failure and continues; a failed
// ASSERT_* records it and returns from the test body; EXPECT_FLOAT_EQ /
// EXPECT_DOUBLE_EQ compare within 4 units in the last place; RUN_ALL_TESTS
// runs every TEST in registration order, prints one line per test and
// returns 1 if any failed.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <sstream>
#include <string>
#include <type_traits>
#include <vector>

namespace testing {

struct TestInfo {
  const char* suite;
  const char* name;
  void (*body)();
};

inline std::vector<TestInfo>& registry() {
  static std::vector<TestInfo> r;
  return r;
}
inline bool& current_failed() {
  static bool f = false;
  return f;
}

struct Registrar {
  Registrar(const char* suite, const char* name, void (*body)()) {
    registry().push_back({suite, name, body});
  }
};

inline void InitGoogleTest(int*, char**) {}
inline void InitGoogleTest() {}

class Message {
 public:
  template <class T>
  Message& operator<<(const T& v) {
    ss_ << v;
    return *this;
  }
  std::string str() const { return ss_.str(); }

 private:
  std::ostringstream ss_;
};

// `Helper(...) = Message() << ...` records the failure; its operator= returns
// void, so an ASSERT can `return` it from a void test body.
class Helper {
 public:
  Helper(const char* file, int line, std::string what)
      : file_(file), line_(line), what_(std::move(what)) {}
  void operator=(const Message& m) const {
    current_failed() = true;
    std::printf("%s:%d: Failure\n  %s\n", file_, line_, what_.c_str());
    const std::string extra = m.str();
    if (!extra.empty()) std::printf("  %s\n", extra.c_str());
  }

 private:
  const char* file_;
  int line_;
  std::string what_;
};

template <class A, class B>
std::string describe(const char* ea, const char* op, const char* eb, const A& a, const B& b) {
  std::ostringstream ss;
  ss << "Expected: (" << ea << ") " << op << " (" << eb << ")";
  if constexpr (requires(std::ostream& o) {
                  o << a;
                  o << b;
                })
    ss << ", actual: " << a << " vs " << b;
  return ss.str();
}

template <class F>
bool almost_equal_ulps(F a, F b) {
  if (std::isnan(a) || std::isnan(b)) return false;
  using I = std::conditional_t<sizeof(F) == 4, std::int32_t, std::int64_t>;
  I ia, ib;
  std::memcpy(&ia, &a, sizeof(F));
  std::memcpy(&ib, &b, sizeof(F));
  // map the sign-magnitude bit patterns onto one ordered integer line
  const I sign = I(1) << (sizeof(F) * 8 - 1);
  ia = ia < 0 ? sign - ia : ia;
  ib = ib < 0 ? sign - ib : ib;
  const auto d = ia > ib ? ia - ib : ib - ia;
  return d <= 4;
}

inline int run_all() {
  int failed = 0;
  for (const TestInfo& t : registry()) {
    current_failed() = false;
    std::printf("[ RUN      ] %s.%s\n", t.suite, t.name);
    t.body();
    std::printf("%s %s.%s\n", current_failed() ? "[  FAILED  ]" : "[       OK ]", t.suite, t.name);
    if (current_failed()) ++failed;
  }
  std::printf("[==========] %zu tests, %d failed\n", registry().size(), failed);
  return failed ? 1 : 0;
}

}  // namespace testing

#define TO_GTEST_CAT2(a, b) a##b
#define TO_GTEST_CAT(a, b) TO_GTEST_CAT2(a, b)

#define TEST(suite, name)                                                                     \
  static void TO_GTEST_CAT(suite, TO_GTEST_CAT(_, TO_GTEST_CAT(name, _body)))();             \
  static ::testing::Registrar TO_GTEST_CAT(suite, TO_GTEST_CAT(_, TO_GTEST_CAT(name, _reg)))( \
      #suite, #name, &TO_GTEST_CAT(suite, TO_GTEST_CAT(_, TO_GTEST_CAT(name, _body))));       \
  static void TO_GTEST_CAT(suite, TO_GTEST_CAT(_, TO_GTEST_CAT(name, _body)))()

#define RUN_ALL_TESTS() ::testing::run_all()

#define TO_GTEST_CHECK_(cond, what, on_fail) \
  if (cond)                                  \
    ;                                        \
  else                                       \
    on_fail ::testing::Helper(__FILE__, __LINE__, what) = ::testing::Message()

#define TO_GTEST_CMP_(a, b, op, on_fail)                                                \
  if (const auto& to_gt_a_ = (a); true)                                                 \
    if (const auto& to_gt_b_ = (b); to_gt_a_ op to_gt_b_)                               \
      ;                                                                                 \
    else                                                                                \
      on_fail ::testing::Helper(__FILE__, __LINE__,                                     \
                                ::testing::describe(#a, #op, #b, to_gt_a_, to_gt_b_)) = \
          ::testing::Message()

#define EXPECT_TRUE(c) TO_GTEST_CHECK_((c), "Expected true: " #c, )
#define EXPECT_FALSE(c) TO_GTEST_CHECK_(!(c), "Expected false: " #c, )
#define ASSERT_TRUE(c) TO_GTEST_CHECK_((c), "Expected true: " #c, return)
#define ASSERT_FALSE(c) TO_GTEST_CHECK_(!(c), "Expected false: " #c, return)

#define EXPECT_EQ(a, b) TO_GTEST_CMP_(a, b, ==, )
#define EXPECT_NE(a, b) TO_GTEST_CMP_(a, b, !=, )
#define EXPECT_LT(a, b) TO_GTEST_CMP_(a, b, <, )
#define EXPECT_LE(a, b) TO_GTEST_CMP_(a, b, <=, )
#define EXPECT_GT(a, b) TO_GTEST_CMP_(a, b, >, )
#define EXPECT_GE(a, b) TO_GTEST_CMP_(a, b, >=, )
#define ASSERT_EQ(a, b) TO_GTEST_CMP_(a, b, ==, return)
#define ASSERT_NE(a, b) TO_GTEST_CMP_(a, b, !=, return)
#define ASSERT_LT(a, b) TO_GTEST_CMP_(a, b, <, return)
#define ASSERT_LE(a, b) TO_GTEST_CMP_(a, b, <=, return)
#define ASSERT_GT(a, b) TO_GTEST_CMP_(a, b, >, return)
#define ASSERT_GE(a, b) TO_GTEST_CMP_(a, b, >=, return)

#define EXPECT_FLOAT_EQ(a, b)                                                                  \
  TO_GTEST_CHECK_(::testing::almost_equal_ulps<float>(static_cast<float>(a),                   \
                                                      static_cast<float>(b)),                  \
                  ::testing::describe(#a, "~=", #b, static_cast<float>(a), static_cast<float>(b)), )
#define EXPECT_DOUBLE_EQ(a, b)                                                      \
  TO_GTEST_CHECK_(::testing::almost_equal_ulps<double>(static_cast<double>(a),      \
                                                       static_cast<double>(b)),     \
                  ::testing::describe(#a, "~=", #b, static_cast<double>(a),         \
                                      static_cast<double>(b)), )
#define EXPECT_NEAR(a, b, tol)                                                      \
  TO_GTEST_CHECK_(std::fabs(static_cast<double>(a) - static_cast<double>(b)) <=     \
                      static_cast<double>(tol),                                     \
                  ::testing::describe(#a, "near", #b, static_cast<double>(a),       \
                                      static_cast<double>(b)), )
#define ASSERT_NEAR(a, b, tol)                                                      \
  TO_GTEST_CHECK_(std::fabs(static_cast<double>(a) - static_cast<double>(b)) <=     \
                      static_cast<double>(tol),                                     \
                  ::testing::describe(#a, "near", #b, static_cast<double>(a),       \
                                      static_cast<double>(b)), return)
