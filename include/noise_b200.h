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

/* Failure-path self-test, no reference counterpart: one launch of the GEMM engine whose producer
 * arms its operand barrier without issuing the copies, with a wait budget of 2e7 cycles (about
 * 10 ms). The MMA warp's bounded wait runs out, the kernel sets *status = NOISE_WAIT_TIMEOUT and ends
 * through its abort path (every role leaves its loop, tensor memory is freed); the context stays
 * usable. A: bf16 [128][64], B: bf16 [256][64] device buffers (never read); returns NOISE_OK when the
 * launch succeeded. */
int noise_selftest_wait_timeout(const void* A, const void* B, int* status, void* stream);

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

/* Workspace bytes for `rows` population rows (rows = members * B * T of one chunk): the per-row
 * activations, the bf16 rotary table and the chunk's draw table (406 KB per direction the chunk
 * spans, for at most min(512, rows / 256 + 2) directions). */
size_t noise_pop_workspace_bytes(int64_t rows);

/* Members per chunk that noise_pop_forward_lowrank (pairs = P) or noise_pop_forward_direct (pairs = 1)
 * processes for `members` members of rows_per_member rows each, given workspace_bytes: the largest
 * chunk whose workspace fits, whose directions fit the draw table and whose rows fit 32-bit GEMM row
 * indices, then evened out so that all chunks have the same size (0: not even one member fits).
 * Sizing the workspace as noise_pop_workspace_bytes(rows_per_member * chunk) gives a buffer that the
 * call uses in full. No reference counterpart (the reference's chunk is the fixed CHUNK = 256 pairs,
 * train/val/eggroll.py:35). */
int noise_pop_chunk_members(int64_t rows_per_member, int members, int pairs, size_t workspace_bytes);

/* Replaces train/val/eggroll.py:66-103 (population_loss, through Eggroll.loss at :115/:145) for
 * members [member_begin, member_begin + members): member j perturbs every parameter by
 * s_j * (a_d b_d^T) (rank-1 factors for matrices and embeddings, eps_d for the mixing scalars) with
 * d = (j mod 2*pairs) / 2 and s_j = +sigma for even j, -sigma for odd j (:134-146). Draw d is
 * regenerated from the Philox stream keyed by (seed, step), once per chunk into the workspace's draw
 * table. Every member evaluates all B rows of
 * tokens/targets ([B, T] int32, T % 128 == 0) and losses[j - member_begin] receives
 * its mean next-token cross-entropy over B*T tokens. rope: [T][64] fp32 = bf16-rounded cos | sin
 * (utils/model.py:177-183). Members are processed in equal chunks that fit `workspace`. */
int noise_pop_forward_lowrank(const float* params, const void* packed, const float* rope, const int32_t* tokens,
                              const int32_t* targets, int B, int T, int64_t member_begin, int members, int pairs,
                              float sigma, uint32_t seed, uint32_t step, float* losses, void* workspace,
                              size_t workspace_bytes, int* status, void* stream);

/* Direct-draw rerun of DUST (train/val/run.py:256-279 DUST.rerun with orthogonal_noise :223-238).
 * Sites (bit k of mask): 0 'transformer.wte' (entry must be -1: rerun from the embedding),
 * 1 'o' (attention output), 2 'attn' (attn.c_proj output), 3 'fc' (mlp.c_fc pre-activation, live
 * units only), 4 'mlp' (mlp.c_proj output). site[k] is the stream id of site k's draws (the
 * parameter tensor id whose output is jittered; hubs o@i use 64 + i; the embedding uses 2). */
typedef struct NoiseDirect {
  int entry;            /* first block rerun, -1 = from the embedding */
  uint32_t mask;        /* sites jittered in block `entry` */
  uint32_t site[5];
  float sigma;          /* jitter scale (draws are +-1) */
  const float* x_entry; /* [B*T, 512] clean input of block `entry` (entry >= 0) */
  const float* inv0;    /* [B*T] clean 1/rms of the embedding rows (entry >= 0) */
  const void* live;     /* bf16 [B*T, 2048] clean relu^2 hidden of block `entry` (fc site) */
  const void* y_entry;  /* optional bf16 [B*T, 512] clean attention output of block `entry` (entry >= 0):
                           when given, block `entry` starts from it (plus the 'o' draw) instead of
                           recomputing its QKV projection and attention, which no site changes */
} NoiseDirect;

/* Replaces DUST.rerun (train/val/run.py:256-279) for draws [draw_begin, draw_begin + draws) of the
 * sites in spec: weights unperturbed, draw i adds sigma * a_i (orthogonal draws regenerated from the
 * (seed, step) stream) at its sites in block `entry`, every draw evaluates all B rows, and
 * token_loss[i - draw_begin][b][t] receives the per-token cross-entropy (0 where targets < 0).
 * entry = -1 with mask = 0 is the plain forward with per-token losses. */
int noise_pop_forward_direct(const float* params, const void* packed, const float* rope, const int32_t* tokens,
                             const int32_t* targets, int B, int T, int64_t draw_begin, int draws,
                             const NoiseDirect* spec, uint32_t seed, uint32_t step, float* token_loss, void* workspace,
                             size_t workspace_bytes, int* status, void* stream);

/* Clean forward of the unperturbed model keeping what DUST's reruns and reassembly need
 * (train/val/run.py:189-209 hooks, capture :244-254). All arrays are caller-owned, rows = B*T. */
typedef struct NoiseCapture {
  float* blocks;      /* [8][rows][512] block inputs after the x0 mixing */
  float* x0;          /* [rows][512] normalised embedding */
  float* inv0;        /* [rows] 1/rms of the embedding rows */
  void* y;            /* bf16 [8][rows][512] attention outputs (c_proj inputs) */
  float* mid;         /* [8][rows][512] residual stream after the attention */
  void* hidden;       /* bf16 [8][rows][2048] relu^2 hidden (mlp.c_proj inputs) */
  float* final_x;     /* [rows][512] residual stream after the last block */
  float* logits;      /* [rows][4096] raw logits before the soft cap */
  float* token_loss;  /* [rows] per-token cross-entropy (0 where targets < 0) */
} NoiseCapture;

int noise_pop_capture(const float* params, const void* packed, const float* rope, const int32_t* tokens,
                      const int32_t* targets, int B, int T, const NoiseCapture* out, void* workspace,
                      size_t workspace_bytes, int* status, void* stream);

/* Credit-memory priors of the sites jittered together in one rerun (train/val/run.py:336-341): mu[s]
 * is [B*T][d[s]] fp32, alpha * M c, masked like the site's draws. */
typedef struct NoisePrior {
  int count;            /* 0, 1 or 2 */
  uint32_t site[2];     /* stream site ids of the draws */
  int d[2];             /* widths (powers of two, <= 2048) */
  const float* mu[2];
} NoisePrior;

/* Replaces the contraction of DUST.direct_errors (train/val/run.py:347-373) for one site: with
 * perturbed [draws][B*T] from noise_pop_forward_direct and clean [B*T], rewards clean - perturbed are
 * centred over chunks of `chunk` consecutive draws, optionally turned into reward-to-go with decay
 * gamma (run.py:81-86), given the centred drop the priors predict (prior may be null), and
 * errors [B*T][d] -= sum_i reward_i a_i / sigma, masked by live (bf16 [B*T][d] > 0) when given.
 * draws <= 2048 per call; the caller divides by the site's total draw count and adds
 * (1 - 1/chunk) mu for a site with a prior. */
int noise_dust_errors(const float* clean, const float* perturbed, int draws, int chunk, int B, int T,
                      int64_t draw_begin, uint32_t site, int d, float sigma, float gamma, const void* live,
                      const NoisePrior* prior, uint32_t seed, uint32_t step, float* errors, void* stream);

/* Replaces coordinate_differences (train/val/run.py:120-137): raw logits [rows][4096] -> the central
 * difference of each token's soft-capped CE along each of its logits, zero where targets < 0. */
int noise_coordinate_differences(const float* raw, const int32_t* targets, int64_t rows, float sigma, float* out,
                                 void* stream);

/* Replaces DUST.reassemble (train/val/run.py:465-471) for a linear site: g[o][i] = sum over the K
 * tokens of err[k][o] * x[k][i] (err fp32 [K][err_ld], x fp32 or bf16 [K][x_ld], g fp32 [out][in]),
 * with x's rows first scaled by 1 / rms(x[k][0 .. x_ld)) when x_norm (the normalised module inputs of
 * mlp.c_fc, lm_head and the attention projections; `in` may be narrower than x_ld, as for ve_gate's
 * first 32 channels). out % 128 == 0, in % 256 == 0 and K % 32 == 0 run on tf32 tensor cores (the
 * reference's float32 einsum under 'high' matmul precision), K split into blocks whose partial
 * products the workspace holds and that are added in order; other shapes in fp32 on CUDA cores. The
 * workspace size depends on the shape only. */
int64_t noise_reassemble_workspace_bytes(int K, int out, int in);
int noise_reassemble(const float* err, int err_ld, int K, int out, const void* x, int x_bf16, int x_ld, int in,
                     int x_norm, float* g, void* workspace, size_t workspace_bytes, int* status, void* stream);

/* DUST's attention-internal errors (replaces DUST.local_errors, train/val/run.py:391-463). One block,
 * one kind: 0 q, 1 k, 2 v, 3 gate, 4 value embedding (3 and 4 on blocks 1, 3, 5, 7 only). All
 * [B*T, 512] operands are bf16 rows of B sequences of T tokens (T % 128 == 0), 16-byte aligned. */
typedef struct NoiseLocal {
  int kind;
  int layer;                /* block: sets the attention window */
  uint32_t site;            /* stream site id of the draws (the tensor id of the site's weight) */
  float sigma;              /* draw scale (0.1) */
  float gamma;              /* lag credit decay per token (0.98) */
  const void* raw;          /* kinds q, k: raw c_q / c_k outputs before RoPE and norm */
  const void* q;            /* processed clean queries: rms_norm(rope(raw q)) per head */
  const void* k;            /* processed clean keys */
  const void* values;       /* clean values v + 2 sigmoid(z) ve */
  const float* gate_logits; /* kinds gate, ve: [B*T][8] fp32 */
  const float* ve;          /* kinds gate, ve: [B*T][512] fp32 value-embedding rows */
  const void* target;       /* the block's hub target */
  const float* base;        /* kinds q, k: [B*T][8] clean scores from noise_local_baseline */
} NoiseLocal;

/* out = bf16(rms_norm(rope(raw))) per head: the reference's `processed` (run.py:405-406). */
int noise_local_process(const void* raw, const float* rope, int B, int T, void* out, void* stream);

/* base[b*T + t][h] = <target, attention(q, k, values)> at (b, t, head h): the clean scores. */
int noise_local_baseline(const NoiseLocal* spec, int B, int T, float* base, int* status, void* stream);

/* Workspace of noise_local_errors for `draws` draws. */
int64_t noise_local_workspace_bytes(int B, int T, int draws);

/* errors [B*T][width] += sum over draws [draw_begin, draw_begin + draws) (draws <= 1024) of the
 * credited score times the draw / divisor (sigma; 2 sigma for the gate); width 8 for the gate, else
 * 512. The caller divides by the total draw count. */
int noise_local_errors(const NoiseLocal* spec, const float* rope, int B, int T, int64_t draw_begin, int draws,
                       uint32_t seed, uint32_t step, float* errors, void* workspace, size_t ws_bytes, int* status,
                       void* stream);

/* A region of the flat parameter layout: tensors [tensor_begin, tensor_end) in named_parameters order,
 * whose optimizer buffers (gradient, moments, ANVIL rails, polar input) are region buffers: their
 * element i holds flat index base + i (base <= the first tensor's flat offset). {0, 60, 0} is the whole
 * buffer. The sharded update gives each rank the region of whole tensors it owns. */
typedef struct NoiseRegion {
  int tensor_begin, tensor_end;
  int64_t base;
} NoiseRegion;

/* Replaces torch.optim.AdamW.step on dense gradients (the DUST estimator's; train/val/run.py:652-655):
 * grad is a full flat gradient buffer; lr_per_tensor[60] gives each tensor's learning rate, < 0
 * for tensors another optimizer owns. adam_t is the 1-based step for the bias corrections. */
int noise_adamw_dense(float* params, void* packed, float* exp_avg, float* exp_avg_sq, const float* grad,
                      const float* lr_per_tensor, float beta1, float beta2, float eps, float weight_decay, int adam_t,
                      void* stream);

/* noise_adamw_dense on one region (params and packed keep the flat layout; exp_avg, exp_avg_sq and grad
 * are region buffers). */
int noise_adamw_region(float* params, void* packed, float* exp_avg, float* exp_avg_sq, const float* grad,
                       const NoiseRegion* region, const float* lr_per_tensor, float beta1, float beta2, float eps,
                       float weight_decay, int adam_t, void* stream);

/* ANVIL II (train/val/run.py:583-626) over the 48 block matrices in named_parameters order, split
 * around `polar` (:572-580), whose quintic maps the caller runs on x as bf16 matmuls. Buffers with
 * the flat parameter layout: grad, fast, slow, scratch (fp32), x (bf16); energy [lanes]; partials
 * [2 * tiles]; scalars [matrices] (sizes from noise_anvil_sizes).
 * prepare: fast/slow EMAs, m = g.lerp(w fast + (1-w) slow, beta), x = bf16(m / (1.05 |m| + 1e-6)).
 * finish: x holds polar(m); lane-energy EMA, normalisation, sign-gated decay, parameter update. */
int noise_anvil_sizes(int64_t* tiles, int64_t* lanes, int* matrices);
int noise_anvil_prepare(const float* grad, float* fast, float* slow, float* scratch, void* x, float* partials,
                        float* scalars, float fast_beta, float slow_beta, float beta, float weight, void* stream);
int noise_anvil_finish(float* params, void* packed, const float* slow, const void* update, float* energy,
                       float* partials, float* scalars, float lane_beta, float lr, float weight_decay, void* stream);

/* ANVIL II's `polar` (train/val/run.py:572-580) on the block matrices of a region, in place on x (the
 * bf16 region buffer noise_anvil_region_prepare wrote): nmaps quintic maps, maps[3k .. 3k+2] = (a, b, c)
 * of map k, X <- a X + (b S + c S S) X with S = X X^T on each matrix's wide form (the transpose of a
 * tall c_fc), batched by shape on the tcgen05 engine in bf16 storage with fp32 accumulation. The
 * workspace holds the stacked matrices (noise_anvil_polar_workspace_bytes; 0 for a region without
 * block matrices). */
int64_t noise_anvil_polar_workspace_bytes(const NoiseRegion* region);
int noise_anvil_region_polar(const NoiseRegion* region, void* x, const float* maps, int nmaps, void* workspace,
                             size_t workspace_bytes, int* status, void* stream);

/* The same three on the block matrices of one region (grad, fast, slow, scratch and x are region
 * buffers; energy, partials and scalars are sized for the region by noise_anvil_region_sizes). */
int noise_anvil_region_sizes(const NoiseRegion* region, int64_t* tiles, int64_t* lanes, int* matrices);
int noise_anvil_region_prepare(const NoiseRegion* region, const float* grad, float* fast, float* slow, float* scratch,
                               void* x, float* partials, float* scalars, float fast_beta, float slow_beta, float beta,
                               float weight, void* stream);
int noise_anvil_region_finish(const NoiseRegion* region, float* params, void* packed, const float* slow,
                              const void* update, float* energy, float* partials, float* scalars, float lane_beta,
                              float lr, float weight_decay, void* stream);

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

/* One rank's share of the reconstruction of train/val/eggroll.py:155-163 for the sharded update
 * (reduce-scatter of partial sums instead of every rank rebuilding all directions, :156-163):
 * g = -grad_scale * sum over d in [dir_begin, dir_begin + dir_count) of weights[d] a_d b_d^T (eps_d for
 * the mixing scalars), every tensor, written to out starting at out_offsets[tensor] (host array of 60;
 * NULL: the flat layout). Summing the outputs of calls over disjoint direction ranges gives the
 * gradient that noise_update_sum_fe_adamw reconstructs. */
int noise_sum_fe_partial(const float* weights, int pairs, int dir_begin, int dir_count, float grad_scale,
                         uint32_t seed, uint32_t step, const int64_t* out_offsets, float* out, void* stream);

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
