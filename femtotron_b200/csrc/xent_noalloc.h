// Allocation-free C entry point: mean cross-entropy loss of bf16 logits.
//
// This entry point has no counterpart in the reference framework; it is an addition of this
// library for callers that cannot allocate GPU memory themselves.
//
// Who needs it: code that must not call cudaMalloc / cudaFree or any allocating library
// routine on its own -- for example a host runtime written in C or another language that
// does not link PyTorch's caching allocator, a process whose device memory is fully reserved
// up front by another allocator, or a call site inside a region where allocation is
// forbidden (allocation can synchronise the device or fail under memory pressure).  Such a
// caller still owns the inputs and the output; the only extra memory this routine needs
// (one float4 of statistics per row) lives in a fixed, file-scope device array of the
// library instead of being allocated per call.
//
// Contract:
//   logits       bf16 [rows, ld] device pointer, 16-byte aligned; the first `vocab` columns of
//                each row are the logits (vocab and ld multiples of 8, ld >= vocab); may be
//                null when rows == 0
//   labels       int64 [rows] device pointer (may be null when rows == 0); rows whose label
//                equals `ignore_index` are skipped; other labels must lie in [0, vocab)
//   loss_out     float [1] device pointer: receives sum(lse - logit[label]) / (#valid rows);
//                NaN when no row is valid (a mean over an empty set) and NaN when any label
//                other than `ignore_index` lies outside [0, vocab), so a broken label shows
//                as NaN instead of a plausible wrong loss
//   stream       cudaStream_t (0 = legacy default stream)
// Returns 0 on success; 1 if rows exceeds FT_XENT_NOALLOC_MAX_ROWS (nothing is launched);
// 2 for an invalid argument; 3 if the one-time device set-up failed; 1000 + cudaError_t if a
// kernel launch failed.
//
// Limits and behaviour:
//   * at most FT_XENT_NOALLOC_MAX_ROWS = 65536 rows per call: the scratch array takes
//     65536 x 16 bytes = 1 MiB on every GPU that loads the library, held until process exit;
//   * the first call on a device looks up the device address of the scratch array
//     (cudaGetSymbolAddress) with that device current; make that first call before any
//     stream capture;
//   * all calls share the one scratch array and each call overwrites the rows it uses, so
//     nothing has to be zeroed between calls -- but calls that overlap on the GPU (on
//     different streams, or from different host threads without ordering) race on it;
//   * it allocates nothing: no cudaMalloc, cudaFree or allocating library routine.
#pragma once

#include <stdint.h>

#define FT_XENT_NOALLOC_MAX_ROWS 65536

#ifdef __cplusplus
extern "C" {
#endif

int ft_xent_mean_loss_noalloc(const void* logits, const int64_t* labels, int64_t rows,
                              int64_t vocab, int64_t ld, int64_t ignore_index, float* loss_out,
                              void* stream);

#ifdef __cplusplus
}
#endif
