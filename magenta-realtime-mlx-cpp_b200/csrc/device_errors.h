// Bits of the per-stream device error word. Kernels set them with
// atomicOr; the host reads and clears the word after each call
// (mrtdf_stream_sync and every synchronous entry point).
#pragma once

namespace mrtdf {

enum : int {
  kErrMbarTimeout = 1 << 0,     // a TMA bulk copy never completed its mbarrier phase
  kErrCounterTimeout = 1 << 1,  // a bounded wait on a counter / flag gave up
  kErrBadToken = 1 << 2,        // a sampled or forced id outside [0, vocab)
  kErrFixedRange = 1 << 3,      // a split-K partial sum beyond the fixed-point range (NaN or |x| >= 2^30)
};

}  // namespace mrtdf
