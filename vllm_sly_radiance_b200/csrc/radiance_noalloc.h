/* C interface of the allocation-free greedy argmax (argmax_noalloc.cu).
 *
 * This entry point has no counterpart in the reference.  It is for callers that cannot allocate
 * device memory when they need a token: a C or C++ host without torch (no caching allocator to
 * draw a workspace from), a process whose KV cache already holds nearly all HBM (a late
 * cudaMalloc may fail), or a decode loop that must not absorb the device-wide synchronisation of
 * cudaMalloc / cudaFree.  Its partials and arrival counters live in one file-scope __device__
 * array per device (about 516 KB, held until the process exits).
 *
 * Library: libradiance_noalloc.so (built beside the package, links only the CUDA runtime); the
 * same symbol is also exported by the torch extension.
 */
#ifndef RADIANCE_NOALLOC_H_
#define RADIANCE_NOALLOC_H_

#ifdef __cplusplus
extern "C" {
#endif

#define RADIANCE_NOALLOC_MAX_ROWS 1024   /* rows per call */
#define RADIANCE_NOALLOC_MAX_CHUNKS 64   /* CTAs per row: any vocabulary size fits */
#define RADIANCE_NOALLOC_MAX_CONTEXTS 64 /* distinct CUDA contexts served per process */

/* Greedy token of each row: out_ids[r] = argmax_j logits[r * ld + j] over j < vocab (ties go to
 * the lowest j), out_vals[r] = that logit (out_vals may be NULL).
 *   logits  : device memory of the current device; dtype 0 = bf16, 1 = fp32
 *   out_ids : device int64[rows]; out_vals: device float[rows] or NULL
 *   stream  : cudaStream_t of the current context (NULL = legacy default stream)
 * Returns 0 on success; otherwise a cudaError_t value (CUDA failure) or -1 (rejected argument:
 * nothing was launched) and, when err is non-NULL, a message in err[0, err_len).
 *
 * The first call in each CUDA context resolves the scratch address; make it before any stream
 * capture begins.  Calls that overlap on one device race on the shared scratch: issue them in
 * order (e.g. all on one stream). */
int radiance_argmax_rows_noalloc(const void* logits, int dtype, int rows, int vocab, long long ld,
                                 long long* out_ids, float* out_vals, void* stream, char* err,
                                 int err_len);

#ifdef __cplusplus
}
#endif

#endif /* RADIANCE_NOALLOC_H_ */
