// Distance kinds of the cuVS API, as declared by the reference
// (include/cuvs/distance/distance.hpp:5-8).  The exact engine accepts
// L2Expanded (squared Euclidean); InnerProduct is declared for source
// compatibility and rejected with std::invalid_argument, as the reference
// rejects it (src/cagra.cpp:26-28).
#pragma once

namespace cuvs::distance {

enum class DistanceType {
  L2Expanded,
  InnerProduct,
};

}  // namespace cuvs::distance
