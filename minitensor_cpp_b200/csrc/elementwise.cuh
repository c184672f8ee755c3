// Host-side planning shared by the precompiled elementwise kernels and the
// runtime-generated fused kernels.
#pragma once

#include "common.cuh"
#include "ew_kernels.cuh"

namespace mtc {

enum class EwVariant { Empty, Flat4, Flat1, Strided, Tiled1, Tiled2, Rows4, Rows1, Tiled4x1, Tiled4x2 };

struct EwPlan {
    MtcEwArgs args;
    EwVariant variant = EwVariant::Empty;
    dim3 grid;
    dim3 block;
};

// Builds the launch plan for `n_out` same-shape outputs computed from `n_in`
// inputs broadcast to that shape.  Validates every descriptor (Float32 only).
int plan_elementwise(const mtc_desc *inputs, int n_in, const mtc_desc *outputs, int n_out, EwPlan &plan);

}  // namespace mtc
