// layout.cuh -- arguments of the layout kernel (see layout.cu).
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace ferryb {

constexpr int kMaxExpertsL = 256;
constexpr int kMaxWorldL = 32;

using LayoutArgs = ferryb_layout_args;  // include/ferryb.h

// ts: device-clock span of the launch (timing mode) or null
int layout_launch(const LayoutArgs& a, cudaStream_t stream, unsigned long long* ts = nullptr);
int layer_slots_launch(const int32_t* slots_row, int capacity, int layer, int experts,
                       int32_t* lookup, cudaStream_t stream);

}  // namespace ferryb
