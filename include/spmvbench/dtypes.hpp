#pragma once
// Value-type traits of the drop-in API (same interface as SpMVBench's
// include/spmvbench/dtypes.hpp): T is the storage type of values and x, Acc
// the accumulator / output type.
#include <cstdint>
#include <type_traits>

namespace spmvbench {

using Index = std::int32_t;

template <typename U>
constexpr bool is_value_type_v = std::is_same_v<U, float> || std::is_same_v<U, double>;

template <typename U>
constexpr const char* dtype_name() {
  static_assert(is_value_type_v<U>, "unsupported value type");
  return std::is_same_v<U, float> ? "fp32" : "fp64";
}

}  // namespace spmvbench
