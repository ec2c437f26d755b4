// The reference keeps device_matrix_view in resources.hpp and this header
// only forwards to it (include/raft/core/device_mdspan.hpp:1-3); same here.
#pragma once

#include <raft/core/resources.hpp>
