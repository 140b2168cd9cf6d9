/* noise_b200 C ABI: the drop-in boundary for Noise's forward-only ES training step on B200.
 *
 * Every entry point takes raw device pointers, sizes and a cudaStream_t (passed as void*), never
 * allocates device memory, and returns an int status (NOISE_OK = 0). Kernels that contain bounded
 * waits also write a status word in device memory (`status`, may be NULL) that the caller reads
 * after synchronising; a nonzero value there means a wait ran out and the outputs are invalid.
 * Launches are asynchronous on `stream`.
 */
#ifndef NOISE_B200_H
#define NOISE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NOISE_OK 0
#define NOISE_BAD_ARGUMENT 1
#define NOISE_LAUNCH_FAILED 2
#define NOISE_WAIT_TIMEOUT 3
#define NOISE_WORKSPACE_TOO_SMALL 4
#define NOISE_UNSUPPORTED 5

/* Engine self-test, no reference counterpart: C[M,N] = alpha * A[M,K] * B[N,K]^T with bf16 A and B
 * (row-major, K contiguous), fp32 accumulation, C stored as bf16 (out_bf16 != 0) or fp32.
 * M % 128 == 0, N % 256 == 0, K % 64 == 0. */
int noise_gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, float alpha, int out_bf16,
                    int* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NOISE_B200_H */
