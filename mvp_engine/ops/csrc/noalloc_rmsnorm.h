// Allocation-free RMSNorm backward: C declaration of the entry point defined in
// noalloc_rmsnorm.cu.  This interface has no counterpart in the reference (MVP
// Engine has no native code); it exists for callers that must not allocate
// device memory while they run kernels: executors that plan every buffer ahead
// of time, code running while a CUDA stream is being captured, real-time
// threads that must not block in an allocator.
//
// Contract (details at the definition):
//   dy, h:  [rows, hidden] bf16, contiguous     rstd: [rows] fp32 (forward 1/RMS)
//   w:      [hidden] bf16                       dx:   [rows, hidden] bf16 (written)
//   dw:     [hidden] fp32 (overwritten)         stream: cudaStream_t or null
//   1 <= hidden <= 16384, hidden % 8 == 0, 1 <= rows <= INT_MAX.
//   Scratch: one 4 MiB file-scope device array per GPU, shared by all calls.
//   Make the first call on each device (it looks up the scratch address)
//   before any stream capture begins.  Calls whose kernels overlap on the GPU
//   race on the scratch; serialise them.  Nothing needs zeroing between calls.
//   Returns 0 on success; 1 too large (nothing launched), 2 bad argument,
//   3 setup failed, 4 launch failed, 5 an earlier CUDA error is pending on this
//   thread (nothing launched, the error is left in place for the caller).
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

int mvp_rmsnorm_bwd_noalloc(const void* dy, const void* h, const float* rstd, const void* w, void* dx, float* dw,
                            int rows, int hidden, void* stream);

#ifdef __cplusplus
}
#endif
