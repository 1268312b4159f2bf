// Attention backward (tcgen05 path) for callers that cannot allocate GPU memory.
//
// This entry point has no counterpart in the reference framework.  It exists for callers
// that must not call cudaMalloc or any allocator: code that runs inside a host allocator
// callback or another library's memory hook (where allocating would recurse or deadlock),
// embedders whose memory is handed out by a fixed arena that the GPU library may not grow,
// and runtimes that forbid allocation on their launch path.  The caller passes the inputs
// and outputs only; the temporary buffers the backward needs (the fp32 dQ accumulator and
// the per-row dot products D = rowsum(dO * O)) live in a fixed file-scope device array of
// REVPP_ATTN_BWD_NOALLOC_SCRATCH_BYTES bytes that every GPU which loads this library holds
// until the process exits.
//
// Shapes and layouts are those of revpp._C.attn_bwd_tc: qkv [B*S, 3H] bf16 (q | k | v,
// H = heads * 64), out and dout [B*S, H] bf16, lse [B, heads, S] fp32, dqkv [B*S, 3H] bf16
// (written).  All pointers are device pointers of the *current* CUDA device; every buffer
// must start on a 16-byte boundary.
//
// Scratch use: 256 bytes (status word) + round_up(B*S*H*4, 256) + B*heads*S*4 bytes must
// fit in REVPP_ATTN_BWD_NOALLOC_SCRATCH_BYTES; larger problems are rejected (return value
// REVPP_NOALLOC_TOO_LARGE, message in `err`) without launching anything.
//
// The first call on a device looks up the scratch array's device address and sets the
// kernel's shared-memory limit for that device; make that first call before any stream
// capture.  Every call on a device shares the same scratch array and overwrites it: two
// calls whose kernels overlap on the GPU (different streams without ordering between
// them) race and give wrong results.  The entry point clears the part of the scratch that
// must start at zero itself, so sequential calls are independent.
//
// `status` (device int, strongly recommended): bits set by the kernels if a bounded wait
// inside them gave up (1 = mbarrier wait); the output is then incomplete.  The caller
// clears the word before the call and reads it after synchronising the stream.  With
// `status == NULL` the bits go to a word inside the scratch array that no caller can read,
// and the return value (which is known before the kernels run) is still REVPP_NOALLOC_OK:
// a caller that passes NULL cannot detect such a failure.  `stream` is a cudaStream_t
// (NULL = legacy default stream).  `err` (optional) receives a message of at most `errlen`
// bytes, NUL-terminated, when the return value is not REVPP_NOALLOC_OK.
#ifndef REVPP_ATTENTION_NOALLOC_H_
#define REVPP_ATTENTION_NOALLOC_H_

#include <stddef.h>

#define REVPP_ATTN_BWD_NOALLOC_SCRATCH_BYTES (16u << 20)

#define REVPP_NOALLOC_OK 0
#define REVPP_NOALLOC_TOO_LARGE 1
#define REVPP_NOALLOC_BAD_ARGUMENT 2
#define REVPP_NOALLOC_CUDA_ERROR 3

#ifdef __cplusplus
extern "C" {
#endif

__attribute__((visibility("default"))) int revpp_attn_bwd_tc_noalloc(
    const void* qkv, const void* out, const void* dout, const float* lse, void* dqkv, int B, int S, int heads,
    int* status, void* stream, char* err, size_t errlen);

#ifdef __cplusplus
}
#endif

#endif  // REVPP_ATTENTION_NOALLOC_H_
