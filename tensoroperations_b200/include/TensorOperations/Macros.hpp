// Macros.hpp -- portable loop-unroll pragma.
#pragma once
#define TENSOR_PRAGMA_UNROLL _Pragma("unroll")
