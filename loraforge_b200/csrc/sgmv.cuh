// Internal interface between the decode SGMV kernels (sgmv.cu) and the prefill
// (tcgen05) SGMV entry point (sgmv_prefill.cu).
#pragma once

#include <stdint.h>

namespace lfb {

enum FusedPhase { kPhaseShrink = 1, kPhaseExpand = 2 };

// Scratch of one decode shrink -> expand call: FP32 partials and z rows (every value
// read is written earlier in the same call) and one completion counter per segment
// (zero before the first call; every call leaves the counters it used at zero).
struct Scratch {
  float* data;
  int* counters;
};

// FP32 elements the decode path needs for these sizes (partials, z rows, counters).
int64_t decode_scratch_floats(int64_t num_tokens, int64_t width, int num_slices, int capacity);

// The decode path's scratch inside a region of decode_scratch_floats(...) floats.
Scratch decode_scratch(float* region, int64_t num_tokens, int64_t width, int num_slices,
                       int capacity);

// The decode shrink -> expand pair over the segments of at most `max_tokens` (<= 16)
// tokens; longer segments are skipped.  Arguments as lf_fused_shrink_expand.
int fused_launch(const void* x, int64_t x_stride, const void* a, const void* b,
                 const int64_t* b_offsets, const int32_t* b_strides, void* y, int64_t y_stride,
                 const int32_t* segment_indptr, const int32_t* segment_slots,
                 const int32_t* token_indices, const int32_t* ranks, const float* scales,
                 const int32_t* slice_offsets, const int32_t* segment_count, const Scratch& scratch,
                 int64_t num_tokens, int64_t width, int32_t out_width, int32_t num_slices,
                 int32_t capacity, int32_t num_slots, int32_t max_segments, int32_t numerics,
                 int max_tokens, void* stream, int phases);

// lf_sgmv_prefill's launches; with z_tok set it runs the shrink only and leaves the FP32 z
// rows by token in z_tok ([num_tokens][rpad], rpad = S*min(capacity, 64) rounded up to 16;
// rows of tokens outside every valid segment are zero).  y is not touched then.
int prefill_launch(const void* x, int64_t x_stride, const void* a, const void* b, const int64_t* b_offsets,
                   const int32_t* b_strides, void* y, int64_t y_stride, const int32_t* segment_indptr,
                   const int32_t* segment_slots, const int32_t* token_indices, const int32_t* ranks,
                   const float* scales, const int32_t* slice_offsets, const int32_t* segment_count,
                   float* workspace, int64_t workspace_floats, int64_t num_tokens, int64_t width,
                   int32_t out_width, int32_t num_slices, int32_t capacity, int32_t num_slots,
                   int32_t max_segments, int32_t numerics, void* stream, float* z_tok);

// Expired bounded waits counted by the prefill kernels' translation unit (synchronous).
int prefill_wait_timeouts(unsigned int* value, int reset);

}  // namespace lfb
