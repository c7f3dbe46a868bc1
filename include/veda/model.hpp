// veda::model — the reference's rotary-position tables and their application outside the tape
// (src/libs/model/Rope.h:41-65), on device tensors: cosines and sines [positions, head_dim] fp32
// from angles computed in double (each written to both halves of the head dimension), and the
// half-split rotation out_i = x_i c - x_{i+p} s, out_{i+p} = x_{i+p} c + x_i s.
#pragma once

#include "veda/tensor.hpp"

#include <cstddef>

namespace veda::model
{

struct RopeTables
{
    core::Tensor cosines;
    core::Tensor sines;
};

// first_position shifts every angle (a query appended after first_position cached positions).
// Throws std::invalid_argument for an odd head_dim.
RopeTables rope_tables(size_t positions, size_t head_dim, float theta, size_t first_position = 0);

// [.., T, Dh] -> [.., T, Dh] rotated, T and Dh matching the tables.
core::Tensor apply_rope(const core::Tensor& x, const RopeTables& tables);

} // namespace veda::model
