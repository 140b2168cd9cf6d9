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
#define NOISE_SCRATCH_LIMIT 6 /* problem larger than a static scratch array holds */

/* Engine self-test, no reference counterpart: C[M,N] = alpha * A[M,K] * B[N,K]^T with bf16 A and B
 * (row-major, K contiguous), fp32 accumulation, C stored as bf16 (out_bf16 != 0) or fp32.
 * M % 128 == 0, N % 256 == 0, K % 64 == 0. */
int noise_gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, float alpha, int out_bf16,
                    int* status, void* stream);

/* Number of fp32 master parameters (37,749,776): one flat buffer in `GPT.named_parameters()` order
 * (utils/model.py:123-147), which is also the `final.pt` state-dict order and the draw-stream tensor
 * id order. */
int64_t noise_param_count(void);

/* Number of bf16 elements of the packed GEMM weights: per block [c_q; c_k; c_v] | c_proj | c_fc |
 * mlp.c_proj, then lm_head. */
int64_t noise_packed_count(void);

/* Refresh the packed bf16 GEMM weights from the fp32 master parameters (the per-matmul bf16 cast
 * that autocast performs in train/val/eggroll.py:144). */
int noise_pack_weights(const float* params, void* packed, void* stream);

/* Workspace bytes for `rows` population rows (rows = members * B * T of one chunk). */
size_t noise_pop_workspace_bytes(int64_t rows);

/* Replaces train/val/eggroll.py:66-103 (population_loss, through Eggroll.loss at :115/:145) for
 * members [member_begin, member_begin + members): member j perturbs every parameter by
 * s_j * (a_d b_d^T) (rank-1 factors for matrices and embeddings, eps_d for the mixing scalars) with
 * d = (j mod 2*pairs) / 2 and s_j = +sigma for even j, -sigma for odd j (:134-146). Draw d is
 * regenerated from the Philox stream keyed by (seed, step). Every member evaluates all B rows of
 * tokens/targets ([B, T] int32, T % 128 == 0) and losses[j - member_begin] receives
 * its mean next-token cross-entropy over B*T tokens. rope: [T][64] fp32 = bf16-rounded cos | sin
 * (utils/model.py:177-183). Members are processed in chunks that fit `workspace`. */
int noise_pop_forward_lowrank(const float* params, const void* packed, const float* rope, const int32_t* tokens,
                              const int32_t* targets, int B, int T, int64_t member_begin, int members, int pairs,
                              float sigma, uint32_t seed, uint32_t step, float* losses, void* workspace,
                              size_t workspace_bytes, int* status, void* stream);

/* Scratch bytes noise_fitness needs for `members` losses. */
size_t noise_fitness_workspace_bytes(int members);

/* Replaces train/val/eggroll.py:151-154. losses[members] (members even; member 2i+1 is the antithetic
 * partner of 2i) -> weights[pairs]. mode 0: z-scored pair differences L[2i+1] - L[2i] over their
 * unbiased std + 1e-8 (the reference); mode 1: differences of centred ranks rank/(N-1) - 0.5 with
 * ranks ascending, NaN last, ties by member index. Pair i contributes to direction i mod pairs.
 * ranks (optional, [members] int32) receives the exact ranks. */
int noise_fitness(const float* losses, int members, int pairs, int mode, float* weights, int32_t* ranks,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Replaces train/val/eggroll.py:155-167 plus torch.optim.AdamW.step (:205): for every parameter
 * tensor g = -grad_scale * sum_d weights[d] a_d b_d^T (eps_d for the mixing scalars), regenerated
 * from the (seed, step) stream, then one AdamW step (lr * lr_mult[tensor] if lr_mult != NULL,
 * betas, eps, decoupled weight_decay, bias corrections for step adam_t) on params/exp_avg/exp_avg_sq,
 * refreshing the packed bf16 copy when packed != NULL. adam_t == 0 only writes g to grad_out
 * (37,749,776 floats, optional otherwise). */
int noise_update_sum_fe_adamw(float* params, void* packed, float* exp_avg, float* exp_avg_sq, const float* weights,
                              int pairs, float grad_scale, uint32_t seed, uint32_t step, const float* lr_mult,
                              float lr, float beta1, float beta2, float eps, float weight_decay, int adam_t,
                              float* grad_out, void* stream);

/* No counterpart in the reference: noise_fitness for callers that cannot allocate device memory
 * (an FFI host with no device allocator of its own, or a process whose device memory another
 * allocator's pool has fully reserved). Same arguments, kernels and results as noise_fitness, but
 * the scratch is a 2 MiB static __device__ array inside the library instead of a caller buffer.
 * Limit: members <= noise_fitness_static_max_members() (262,144); larger calls return
 * NOISE_SCRATCH_LIMIT. The first call on a device looks up the array's address (make it before any
 * stream capture). All calls share the array: calls that overlap on the GPU race, so serialise them
 * on one stream. */
int noise_fitness_static_max_members(void);
int noise_fitness_static(const float* losses, int members, int pairs, int mode, float* weights, int32_t* ranks,
                         void* stream);

/* Instrumentation, no reference counterpart: total kernel launches made by this library so far;
 * optional per-kind device timing with CUDA events recorded on the launching stream (kinds: 0 embed,
 * 1 qkv, 2 attention, 3 proj, 4 fc, 5 mlp, 6 head, 7 loss, 8 fitness, 9 update, 10 pack, 11 other).
 * noise_profile_read synchronises on the recorded events and sums per kind. */
int64_t noise_launch_count(void);
int noise_profile_enable(int on);
int noise_profile_read(double* ms, int64_t* count, int kinds);

#ifdef __cplusplus
}
#endif

#endif /* NOISE_B200_H */
