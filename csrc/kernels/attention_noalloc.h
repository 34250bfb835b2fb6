// Allocation-free flash-attention backward: exported C symbols.
//
// These entry points have no counterpart in the reference implementation.
// They serve callers that cannot allocate device memory at call time (C or
// other-language callers without a CUDA allocator, fixed-budget deployments
// that forbid allocation after set-up, code where cudaMalloc is not allowed).
// Scratch lives in a 16 MiB static device array inside this library; the
// definitions in attention_noalloc.cu state the size rule, the first-call-
// before-stream-capture rule (the first call on a device resolves the scratch
// array and the status word), and that overlapping calls on one device race.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

// Bytes of static scratch available to one call (delta + aligned dQ accumulator).
unsigned long long uhfs_flash_attn_bwd_noalloc_capacity(void);

// Message of the last failed call made by the calling host thread ("" after success).
const char* uhfs_flash_attn_bwd_noalloc_error(void);

// First error code recorded in the current device's status word by a kernel
// whose bounded wait ran out (0 = none); clears it when `clear` != 0.  Call
// after the stream has finished; -1 if the word cannot be read.
int uhfs_flash_attn_bwd_noalloc_status(int clear);

// Backward of multi-head attention over a fused [B*T, 3*H*D] bf16 QKV matrix.
// Returns 0 ok, 1 invalid arguments, 2 problem larger than the static scratch,
// 3 CUDA error.  `stream` is a cudaStream_t (0 = legacy default stream).
int uhfs_flash_attn_bwd_noalloc(const void* qkv, const void* o, const float* lse, const void* dout, void* dqkv,
                                int B, int T, int H, int D, float scale, int causal, void* stream);

#ifdef __cplusplus
}
#endif
