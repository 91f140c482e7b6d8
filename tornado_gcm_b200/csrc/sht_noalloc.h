// Allocation-free spherical-harmonic synthesis (C ABI).
//
// This entry point has no counterpart in the reference.  It exists for
// callers that must not allocate device memory while they run: code that
// owns a fixed memory budget (a runtime with its own arena, an embedded
// solver), code that runs where the CUDA caching allocator of PyTorch is not
// present or must not grow, and plain C callers that have no allocator at
// all.  The regular synthesis op takes its intermediate buffer from PyTorch;
// this one keeps it in a fixed array compiled into the library.
//
// What it computes is the regular synthesis op of the extension, modal
// (S, 2M-1, L) -> nodal (S, I, J) (or (S, J, I) with lat_major != 0), with
// the same two tcgen05 TF32 GEMMs (Legendre, then Fourier).
//
// Limits and sharing:
// * The intermediate needs S * J * M2p floats, at most
//   TGCM_SHT_NOALLOC_SCRATCH_FLOATS (4 Mi floats = 16 MiB).  Larger requests
//   are rejected with TGCM_SHT_NOALLOC_ERR_TOO_LARGE and a message on stderr;
//   split the S slices over several calls instead.
// * The 16 MiB array is static device memory: every GPU on which the
//   library's device code is loaded holds it until the process exits.
// * All calls share that one array.  Two calls whose kernels overlap on the
//   GPU (different streams, or different host threads on one device) race on
//   it and give wrong results: order them on one stream or synchronise.
//   Each call writes every scratch element it later reads, so no part of the
//   array has to start at zero and the previous call's contents do no harm.
// * The first call on each device performs a one-time set-up for that
//   device (looks up the array's device address, sets the kernels' shared
//   memory limit).  Make that first call before any stream capture on the
//   device, e.g. with a small warm-up call.
// * Nothing here allocates: no cudaMalloc / cudaFree, no PyTorch, no
//   heap-backed containers.  Tensor maps are built on the stack per call.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TGCM_SHT_NOALLOC_SCRATCH_FLOATS (4u * 1024u * 1024u)

#define TGCM_SHT_NOALLOC_OK 0
#define TGCM_SHT_NOALLOC_ERR_ARGS 1       // shape, stride or alignment not supported
#define TGCM_SHT_NOALLOC_ERR_TOO_LARGE 2  // S * J * M2p above TGCM_SHT_NOALLOC_SCRATCH_FLOATS
#define TGCM_SHT_NOALLOC_ERR_CUDA 3       // a CUDA runtime / driver call failed (message on stderr)

// Arguments (all pointers are device pointers on the current device):
//   x        modal input, S slices of M2 = 2*Mw-1 rows of L floats; element
//            (s, r, l) at x[s * x_slice_stride + r * x_row_stride + l].
//            16-byte aligned; both strides multiples of 4 floats.
//   P        Legendre table (Mw, J, Lp) contiguous, Lp >= L, Lp % 4 == 0.
//            It must be lower-triangular in the sense of the associated
//            Legendre functions: P[m, j, l] == 0 for l < m.  The Legendre
//            GEMM of group m starts its K loop at floor(m / 32) * 32 and
//            skips the columns before it, so non-zero entries there would be
//            dropped.  For the same reason every group must have at least
//            one K block: floor((Mw - 1) / 32) * 32 < L, which holds for
//            every spectral truncation with Mw <= L.  Calls that break it are
//            rejected with TGCM_SHT_NOALLOC_ERR_ARGS.
//   F        real Fourier table (I, M2p) contiguous, M2p >= M2, M2p % 4 == 0.
//   out      nodal output, contiguous (S, I, J), or (S, J, I) when lat_major.
//   err      optional int flag (device memory, caller sets it to 0); a bounded
//            wait that expires inside a kernel writes a non-zero code there.
//            May be NULL.
//   stream   stream to launch on (0 = legacy default stream).
// Returns one of the TGCM_SHT_NOALLOC_* codes.  TGCM_SHT_NOALLOC_ERR_ARGS
// and TGCM_SHT_NOALLOC_ERR_TOO_LARGE are decided before anything is
// launched.  On TGCM_SHT_NOALLOC_ERR_CUDA the first (Legendre) GEMM may
// already be queued on the stream and writing the shared scratch array when
// the second launch is the one that failed; `out` is then not valid.
int tgcm_sht_synth_noalloc(const float* x, long long S, long long M2, long long L, long long x_row_stride,
                           long long x_slice_stride, const float* P, long long Mw, long long J, long long Lp,
                           const float* F, long long I, long long M2p, float* out, int lat_major, int* err,
                           cudaStream_t stream);

#ifdef __cplusplus
}
#endif
