// Causal sliding-window prefill on the sm_100a tensor cores (tcgen05 + TMEM).
// Placeholder dispatch until the tensor-core kernel lands: no shape is routed here.
#pragma once

#include "prefill_generic.cuh"

namespace spa {

inline bool prefill_sm100_supported(const PrefillArgs&, int) { return false; }

template <typename T>
int launch_prefill_sm100(const PrefillArgs& a, int, cudaStream_t st) {
  return launch_prefill_generic<T>(a, st);
}

}  // namespace spa
