// Allocation-free entry point: pack + Frobenius normalisation factor.
//
// This entry point has no counterpart in the reference (muonium). It exists
// for callers that cannot allocate GPU memory at the point they call us: code
// running inside a custom allocator or memory-pool callback (where a nested
// cudaMalloc would re-enter the allocator), runtimes that own all device
// memory up front and forbid further allocations, and plain C hosts that link
// the library without PyTorch and therefore have no caching allocator.
//
// It runs the same two kernels as the PyTorch binding pair
// muon_pack (without momentum) + norm_finalize, but keeps the per-tile partial
// sums and the per-matrix source-pointer table in one file-scope device array
// of fixed size (kNoAllocScratchBytes, about 4 MiB, held by every GPU that loads
// the library until the process exits). The caller passes the input and both
// outputs.
//
// Limits: batch <= kNoAllocMaxBatch and batch * (Np/64) * (Mp/64) <=
// kNoAllocMaxPartials; larger problems are rejected with an error code.
//
// Set-up: the first call on each device looks up the device address of the
// scratch array (cudaGetSymbolAddress) with that device current, so make the
// first call on a device before any stream capture begins.
//
// Concurrency: every call shares the one scratch array. Calls whose kernels
// may overlap on the GPU (different streams, or different host threads without
// ordering) race on it; serialise them on one stream. Nothing in the scratch
// needs to start at zero: each call overwrites every entry it reads.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  kNoAllocMaxBatch = 1024,
  kNoAllocMaxPartials = 1 << 20,
};

// src:       contiguous [batch, R, C] matrices, fp32 (src_dtype 0) or bf16 (1).
// out_ws:    bf16 [batch, Np, Mp] workspace, Np >= min(R,C), Mp >= max(R,C),
//            both multiples of 64; receives the (transposed when R > C)
//            zero-padded bf16 copy.
// inv_norm:  fp32 [batch]; receives 1 / (||X_b||_F * fac + eps).
// Returns 0 on success, a cudaError_t value from set-up or launch, or -1 for
// arguments outside the documented limits. Launch errors are read with
// cudaPeekAtLastError, so the thread's error state is left untouched, and a
// nonzero value may be an earlier, still pending error of the caller's own.
int dmb_pack_normalize_noalloc(const void* src, int src_dtype, int batch, int R, int C, int Np, int Mp,
                               float fac, float eps, void* out_ws, float* inv_norm, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
