// layout.cuh -- arguments of the layout kernel (see layout.cu).
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace ferryb {

constexpr int kMaxExpertsL = 256;
constexpr int kMaxWorldL = 32;

using LayoutArgs = ferryb_layout_args;  // include/ferryb.h

// Host mirror of the plan summary (the executor's one host wait): pinned,
// mapped host memory that the layout kernel fills at its end -- the summary,
// the executor's eight device error words -- and then releases by writing
// `seq` (system scope), which the host polls.
struct SummaryMirror {
  ferryb_layout_summary* sum;  // device pointer of the mapped host struct, or null (no mirror)
  int32_t* errs;               // mapped [8]
  uint64_t* seq;               // mapped [1]
  const int32_t* errs_dev;     // the executor's error words [8]
  uint64_t value;              // written to *seq last
};

// ts: device-clock span of the launch (timing mode) or null
int layout_launch(const LayoutArgs& a, cudaStream_t stream, unsigned long long* ts = nullptr,
                  const SummaryMirror* mirror = nullptr);
int layer_slots_launch(const int32_t* slots_row, int capacity, int layer, int experts,
                       int32_t* lookup, cudaStream_t stream);

}  // namespace ferryb
