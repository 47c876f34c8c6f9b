// gtest.h -- the few GoogleTest assertion macros that the reference's
// contract headers use (tests/cpp/profiling_contract.hpp and
// decode_batch_contract.hpp in the reference tree), so that those contracts
// compile into adapter_contract without
// GoogleTest, which this image does not have.  A failed assertion prints its
// place and is counted; ASSERT_* also returns from the enclosing function, as
// GoogleTest's does.
#pragma once

#include <cstdio>

namespace gtest_shim {
inline int& failures() {
  static int n = 0;
  return n;
}
inline void fail(const char* file, int line, const char* what) {
  ++failures();
  std::printf("FAIL %s:%d %s\n", file, line, what);
}
}  // namespace gtest_shim

#define EXPECT_TRUE(c)                                                   \
  do {                                                                   \
    if (!(c)) ::gtest_shim::fail(__FILE__, __LINE__, "EXPECT_TRUE(" #c ")"); \
  } while (0)
#define EXPECT_FALSE(c) EXPECT_TRUE(!(c))
#define EXPECT_EQ(a, b) EXPECT_TRUE((a) == (b))
#define EXPECT_NE(a, b) EXPECT_TRUE((a) != (b))
#define EXPECT_GE(a, b) EXPECT_TRUE((a) >= (b))
#define EXPECT_LE(a, b) EXPECT_TRUE((a) <= (b))
#define EXPECT_NEAR(a, b, tol) EXPECT_TRUE(((a) > (b) ? (a) - (b) : (b) - (a)) <= (tol))
#define ASSERT_TRUE(c)                                                    \
  do {                                                                    \
    if (!(c)) {                                                           \
      ::gtest_shim::fail(__FILE__, __LINE__, "ASSERT_TRUE(" #c ")");      \
      return;                                                             \
    }                                                                     \
  } while (0)
#define ASSERT_FALSE(c) ASSERT_TRUE(!(c))
#define ASSERT_EQ(a, b) ASSERT_TRUE((a) == (b))
