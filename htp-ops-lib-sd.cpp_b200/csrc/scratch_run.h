// Internal interface between capi.cu and noalloc.cu: the W8A8 run on a
// caller-owned, fixed scratch array (used by htpg_w8a8_run_static).
#pragma once
#include <cstddef>

#include "../../include/htp_ops_b200.h"

namespace htpg {

// Bytes at the start of the scratch array reserved for split-K partial sums
// and tile counters (128 weight tiles x 128 rows x 32 rows of INT32 + 4 KiB).
constexpr size_t kStaticSplitKBytes = 128u * 128u * 32u * 4u + 4096u;

// htpg_w8a8_run with its activation codes, row scales and split-K area in
// [scratch, scratch + scratch_bytes); HTPG_ESCRATCH when they do not fit.
int w8a8_run_in_scratch(const htpg_weights *w, float *out, int ldo, const float *x, const float *bias,
                        int m, int channels, int mode, void *stream, void *scratch, size_t scratch_bytes);

// Sets the text htpg_last_cuda_error returns on this thread.
void set_error_text(const char *text);

}  // namespace htpg
