// gtest_main.cpp -- TEST INFRASTRUCTURE: the main() a reference unit test file
// without its own gets (GoogleTest's gtest_main, with Kokkos initialised as
// the reference's test files that do define main() initialise it).
#include <Kokkos_Core.hpp>
#include <gtest/gtest.h>

int main(int argc, char* argv[]) {
  ::testing::InitGoogleTest(&argc, argv);
  Kokkos::initialize(argc, argv);
  const int result = RUN_ALL_TESTS();
  Kokkos::finalize();
  return result;
}
