/*
 * pgf.h -- C-ABI of the B200 (sm_100a) PGF training-step library, libpgf.so.
 *
 * The reference (zhry915/icml) is pure Python: it has no FFI of its own.  Each entry point
 * below replaces one block-streamed operator of its Python modules; the citation next to each
 * names the reference function whose arguments and results it reproduces.  The Python
 * modules in icml_b200/ keep the reference signatures and call these through ctypes.
 *
 * Conventions
 *  - All tensor arguments are device pointers to contiguous row-major buffers; sizes are
 *    element counts.  `dtype` selects the activation type (PGF_DTYPE_F32 or PGF_DTYPE_BF16);
 *    parameters and parameter gradients are always float32, gradients accumulate in float32.
 *  - Every call is stream-ordered on `stream` (a cudaStream_t), never synchronises, never
 *    allocates device memory: scratch comes from the caller through (`ws`, `ws_bytes`), sized
 *    by the matching *_workspace() function.
 *  - Return value: PGF_OK (0) or a PGF_ERR_* code; pgf_last_error() (thread-local) describes
 *    the last failure.  Nothing aborts, throws or exits.
 *  - `accumulate` = 1 adds parameter gradients into the output buffers instead of overwriting.
 *  - Results are deterministic: no floating-point atomics; reductions run in a fixed order.
 */
#ifndef PGF_H_
#define PGF_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PGF_OK 0
#define PGF_ERR_INVALID 1
#define PGF_ERR_CUDA 2
#define PGF_ERR_WORKSPACE 3
#define PGF_ERR_UNSUPPORTED 4

#define PGF_DTYPE_F32 0
#define PGF_DTYPE_BF16 1

/* activation codes: FFN (pgf_ffn.py:81-88) and SSM output activation
   (train_singlemamba_optimized.py:103-114) */
#define PGF_ACT_NONE 0
#define PGF_ACT_GELU 1
#define PGF_ACT_RELU 2
#define PGF_ACT_TANH 3

typedef void* pgf_stream_t; /* cudaStream_t */

/* Last error message of the calling thread ("" if none). */
const char* pgf_last_error(void);
/* Library version, major*10000 + minor*100 + patch. */
int pgf_version(void);

/* Instrumentation (no counterpart in the reference, which has no native code).
 * pgf_launch_count: number of kernels this library has launched in the process.
 * pgf_profile(1) starts recording a CUDA-event pair around each launch of the kernels listed in
 * PGF_PROF_* (stream-ordered, no synchronisation); pgf_profile(0) stops.  pgf_profile_read
 * synchronises on the recorded events and returns, for one kernel since the last pgf_profile(1),
 * its launch count, summed device time and summed algorithmic work: FLOPs (2*M*N*K) for the dense
 * products, bytes that must cross HBM at least once for the bandwidth kernels. */
#define PGF_PROF_SSM_CHUNK_FWD 0
#define PGF_PROF_SSM_COMPOSE 1
#define PGF_PROF_SSM_OUT_FWD 2
#define PGF_PROF_SSM_CHUNK_BWD 3
#define PGF_PROF_SSM_MAIN_BWD 4
#define PGF_PROF_GEMM_TC 5
#define PGF_PROF_GEMM_SIMT 6
#define PGF_PROF_RMSNORM_FWD 7
#define PGF_PROF_RMSNORM_BWD 8
#define PGF_PROF_EMBEDDING 9
#define PGF_PROF_CE 10 /* the fused LM-head + cross-entropy tensor-core passes */
#define PGF_PROF_OPTIM 11 /* pgf_adamw_step */
long long pgf_launch_count(void);
/* Reads and clears the fault flag of the tensor-core engine: 1 if a bounded mbarrier wait expired
 * in a tcgen05 kernel since the last call (the kernel then skipped its epilogue and returned).
 * Synchronous; -1 if the flag cannot be read. */
int pgf_tc_fault(void);
int pgf_profile(int enable);
int pgf_profile_read(int id, long long* count, double* total_ms, double* total_work);

/* ------------------------------------------------------------------------------------------
 * RMSNorm.  Replaces RMSNorm.pgf_forward (pgf_rmsnorm.py:89-117, math :10-18) and
 * RMSNorm.pgf_grad (pgf_rmsnorm.py:157-214, math :22-51).
 *   y = x / sqrt(mean(x^2) + eps) * weight                      x, y: (rows, dim)
 *   grad_weight = sum_rows g * x / rms;  grad_x = g*w/rms - x * sum(g*w*x) / (rms^3 * dim)
 * ------------------------------------------------------------------------------------------ */
int pgf_rmsnorm_fwd(const void* x, const float* weight, void* y, int64_t rows, int64_t dim,
                    float eps, int dtype, pgf_stream_t stream);
/* The block's residual sum and its norm in one pass (pgf_mamba_block.py:109-112, `y + x` then
 * norm2): sum_out = x + res (stored in dtype), y = RMSNorm(sum_out) * weight.  Same bits as the
 * separate add followed by pgf_rmsnorm_fwd.  sum_out must not alias x or res. */
int pgf_rmsnorm_fwd_res(const void* x, const void* res, const float* weight, void* sum_out, void* y,
                        int64_t rows, int64_t dim, float eps, int dtype, pgf_stream_t stream);
size_t pgf_rmsnorm_bwd_workspace(int64_t rows, int64_t dim);
int pgf_rmsnorm_bwd(const void* x, const void* g, const float* weight, void* grad_x /* nullable */,
                    float* grad_weight, int accumulate, int64_t rows, int64_t dim, float eps,
                    int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
/* pgf_rmsnorm_bwd with the skip connection's gradient added to grad_x (pgf_mamba_block.py:202,
 * :246-249, `norm.grad_x + g`): grad_x = RMSNorm'(x)^T g + g_add, with the first term rounded to
 * dtype first, so the bits match the separate add. */
int pgf_rmsnorm_bwd_add(const void* x, const void* g, const float* weight, const void* g_add, void* grad_x,
                        float* grad_weight, int accumulate, int64_t rows, int64_t dim, float eps, int dtype,
                        void* ws, size_t ws_bytes, pgf_stream_t stream);
/* Same results as pgf_rmsnorm_bwd, for callers that cannot allocate device memory (an engine that
 * owns all device memory and forbids allocation from its operators, or a loop that must not enter
 * the allocator).  No counterpart in the reference, which has no native layer.  Scratch is a 4 MiB
 * static device array inside libpgf.so instead of `ws`: the call is rejected (PGF_ERR_INVALID) when
 * dim > 4096 or ceil(rows/32)*dim > 1048576.  Each call looks up the array's address in the calling
 * thread's current CUDA context (the address belongs to that context); the first call in a context
 * may load the library's device code, so make it before any stream capture.  rows = 0 sets
 * grad_weight to zero (leaves it unchanged with accumulate).  All calls share the array: calls that
 * overlap on the GPU race; serialise them. */
int pgf_rmsnorm_bwd_noalloc(const void* x, const void* g, const float* weight,
                            void* grad_x /* nullable */, float* grad_weight, int accumulate,
                            int64_t rows, int64_t dim, float eps, int dtype, pgf_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Embedding.  Replaces pgf_embedding_forward (pgf_embedding.py:74-124) and
 * pgf_embedding_grad (pgf_embedding.py:14-71).  The gradient is a deterministic
 * sort-by-id then segment-sum (the reference's index_add_ is atomic on CUDA).
 *   ids: (n_tokens,) int64 in [0, vocab);  weight, grad_weight: (vocab, dim) float32;
 *   y, g: (n_tokens, dim) in `dtype`.
 * ------------------------------------------------------------------------------------------ */
int pgf_embedding_fwd(const int64_t* ids, const float* weight, void* y, int64_t n_tokens,
                      int64_t vocab, int64_t dim, int dtype, pgf_stream_t stream);
size_t pgf_embedding_bwd_workspace(int64_t n_tokens, int64_t vocab, int64_t dim);
int pgf_embedding_bwd(const int64_t* ids, const void* g, float* grad_weight, int accumulate,
                      int64_t n_tokens, int64_t vocab, int64_t dim, int dtype, void* ws,
                      size_t ws_bytes, pgf_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Dense product with fused epilogue (the matmuls of pgf_ffn.py:43-53, 90-112,
 * pgf_lm_head.py:20-40 and train_singlemamba_optimized.py:120, 440-461).
 *   D[m,n] = epi( alpha * sum_k opA[m,k] * opB[n,k] )
 *   opA[m,k] = a_trans ? A[k*lda + m] : A[m*lda + k]       (M x K)
 *   opB[n,k] = b_trans ? B[k*ldb + n] : B[n*ldb + k]       (N x K, i.e. nn.Linear weight layout)
 * Epilogue order: v = alpha*acc (+ bias[n]); GELU/RELU: aux_out[m,n] = v (if given), v = act(v);
 * DGELU/DRELU: v *= act'(aux[m,n]); v += addend[m,n] (if given); v += D[m,n] (if accumulate).
 * ------------------------------------------------------------------------------------------ */
#define PGF_EPI_NONE 0
#define PGF_EPI_GELU 1
#define PGF_EPI_RELU 2
#define PGF_EPI_DGELU 3
#define PGF_EPI_DRELU 4

typedef struct pgf_epilogue {
  int kind;
  float alpha;
  const float* bias;      /* (N,) or NULL */
  const void* aux;        /* DGELU/DRELU pre-activation (M x N) */
  int aux_dtype;
  int64_t ld_aux;
  void* aux_out;          /* GELU/RELU: pre-activation output (M x N) or NULL */
  int aux_out_dtype;
  int64_t ld_aux_out;
  const void* addend;     /* (M x N) or NULL */
  int addend_dtype;
  int64_t ld_addend;
  int accumulate;         /* D must be float32 */
} pgf_epilogue;

int pgf_gemm(int64_t M, int64_t N, int64_t K, const void* A, int a_dtype, int64_t lda, int a_trans,
             const void* B, int b_dtype, int64_t ldb, int b_trans, void* D, int d_dtype,
             int64_t ldd, const pgf_epilogue* epi, pgf_stream_t stream);

/* pgf_gemm with split-K scratch.  When the (M x N) output has too few tiles to occupy every SM
   (weight gradients, whose depth K is the token count), K is cut into slices that run in
   parallel; their float32 partial products go to `ws` and are summed in slice order
   (deterministic) before the epilogue.  ws_bytes >= pgf_gemm_workspace(M, N, K); a smaller
   scratch (or none) runs the product unsplit. */
size_t pgf_gemm_workspace(int64_t M, int64_t N, int64_t K);
int pgf_gemm_ex(int64_t M, int64_t N, int64_t K, const void* A, int a_dtype, int64_t lda, int a_trans,
                const void* B, int b_dtype, int64_t ldb, int b_trans, void* D, int d_dtype,
                int64_t ldd, const pgf_epilogue* epi, void* ws, size_t ws_bytes, pgf_stream_t stream);

/* Column sums: out[n] (+)= sum_m X[m*ld + n]; deterministic (fixed-order two-level sum).
   The bias gradients of pgf_ffn.py:95,109 and train_singlemamba_optimized.py:443. */
size_t pgf_colsum_workspace(int64_t M, int64_t N);
int pgf_colsum(const void* X, int dtype, int64_t M, int64_t N, int64_t ld, float* out,
               int accumulate, void* ws, size_t ws_bytes, pgf_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * FFN.  Replaces pgf_ffn_forward (pgf_ffn.py:261-307, block math :34-55) and pgf_ffn_grad
 * (pgf_ffn.py:183-258, block math :58-117 with the missing grad_W1 = grad_z^T x).
 *   y = act(x W1^T + b1) W2^T + b2, x: (rows, d_in), W1: (d_hidden, d_in), W2: (d_out, d_hidden).
 * Rows are processed in tiles so the workspace stays bounded by the tile, not by rows.
 * ------------------------------------------------------------------------------------------ */
size_t pgf_ffn_workspace(int64_t rows, int64_t d_in, int64_t d_hidden, int64_t d_out, int dtype,
                         int backward);
int pgf_ffn_fwd(const void* x, const float* W1, const float* b1, const float* W2, const float* b2,
                void* y, int64_t rows, int64_t d_in, int64_t d_hidden, int64_t d_out,
                int activation, int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
/* pgf_ffn_fwd plus a residual in the activation dtype, added in the second product's epilogue and
 * rounded once: y = FFN(x) + res, the block's `ffn(norm2(x1)) + x1` (pgf_mamba_block.py:120-126)
 * without a separate add over the activations. */
int pgf_ffn_fwd_res(const void* x, const float* W1, const float* b1, const float* W2, const float* b2,
                    const void* res, void* y, int64_t rows, int64_t d_in, int64_t d_hidden, int64_t d_out,
                    int activation, int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
int pgf_ffn_bwd(const void* x, const void* g, const float* W1, const float* b1, const float* W2,
                float* grad_W1, float* grad_b1, float* grad_W2, float* grad_b2,
                void* grad_x /* nullable */, int accumulate, int64_t rows, int64_t d_in,
                int64_t d_hidden, int64_t d_out, int activation, int dtype, void* ws,
                size_t ws_bytes, pgf_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * LM head.  pgf_lm_head_forward (pgf_lm_head.py:96-130): logits (float32, T x V) = h W^T.
 * pgf_lm_head_grad (pgf_lm_head.py:45-93): grad_W = g^T h, grad_h = g W.
 * ------------------------------------------------------------------------------------------ */
size_t pgf_lm_head_workspace(int64_t T, int64_t V, int64_t d, int dtype);
int pgf_lm_head_fwd(const void* h, const float* W, float* logits, int64_t T, int64_t V, int64_t d,
                    int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
int pgf_lm_head_bwd(const void* h, const float* g_logits, const float* W, float* grad_W,
                    void* grad_h /* nullable */, int accumulate, int64_t T, int64_t V, int64_t d,
                    int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);

/* LM head fused with the mean cross entropy of test_multi_layer_grads.py:74-86 /
 * train_wikitext_rebuttal.py:116-125, tiled over tokens and vocabulary: the (T x V) logits and
 * their gradient exist only one (token tile x vocab tile) at a time.
 *   fwd: loss_rows[t] = lse_t - logit[t, target_t], lse[t] = logsumexp_v logit[t, v].
 *   bwd: g = (softmax - onehot(target)) * grad_scale; grad_W (+)= g^T h; grad_h = g W.
 * A target outside [0, V) gives that row a NaN loss (the reference's F.cross_entropy raises; these
 * calls do not synchronise to report it). */
size_t pgf_lm_head_ce_workspace(int64_t T, int64_t V, int64_t d, int dtype);
int pgf_lm_head_ce_fwd(const void* h, const float* W, const int64_t* targets, float* loss_rows,
                       float* lse, int64_t T, int64_t V, int64_t d, int dtype, void* ws,
                       size_t ws_bytes, pgf_stream_t stream);
int pgf_lm_head_ce_bwd(const void* h, const float* W, const int64_t* targets, const float* lse,
                       float grad_scale, float* grad_W, void* grad_h, int accumulate, int64_t T,
                       int64_t V, int64_t d, int dtype, void* ws, size_t ws_bytes,
                       pgf_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Selective-scan layer of SingleLayerMambaPGF (train_singlemamba_optimized.py:88-472).
 * Parameters: W_cat = [dt_proj.weight; B_proj.weight; C_proj.weight] (D+2N, D),
 * b_cat (D+2N,), A_log (N,), Dp = D (D,), scale (D,).  u, y, g, grad_u: (Bsz, L, D) in dtype.
 *
 * pgf_ssm_fwd: project (:116-124), discretise (:140-144), scan (:41-52), output map
 *   y = (act(sum_n C h) + Dp*u) * scale (pgf_mamba_block.py:86-112), starting from h_init
 *   (NULL = zeros).  h_final (nullable) receives the state after the last token.
 * pgf_ssm_bwd: _pass2_block_direct_grad (:350-472) over the whole range [0, L): recompute from
 *   h_init, reverse adjoint scan seeded by (dh_end, dA_end) (NULL = zeros / ones), all
 *   parameter gradients and grad_u.  dh_start / dA_start (nullable) return the reference's
 *   (delta_h_block[0], dA[0]).  grad_scale is the per-channel gradient sum(g*y_raw) over
 *   (batch, time) -- autograd's value for the (D,) parameter; the reference's scalar
 *   (:400) is recovered by summing it.
 * N must be 16.  act in {NONE, RELU, TANH}.
 * ------------------------------------------------------------------------------------------ */
size_t pgf_ssm_workspace(int64_t Bsz, int64_t L, int64_t D, int64_t N, int dtype, int backward);
int pgf_ssm_fwd(const void* u, const float* W_cat, const float* b_cat, const float* A_log,
                const float* Dp, const float* scale, const float* h_init, void* y,
                float* h_final, int64_t Bsz, int64_t L, int64_t D, int64_t N, int act, int dtype,
                void* ws, size_t ws_bytes, pgf_stream_t stream);
int pgf_ssm_bwd(const void* u, const void* g, const float* W_cat, const float* b_cat,
                const float* A_log, const float* Dp, const float* scale, const float* h_init,
                const float* dh_end, const float* dA_end, float* grad_W_cat, float* grad_b_cat,
                float* grad_A_log, float* grad_Dp, float* grad_scale, void* grad_u,
                float* dh_start, float* dA_start, int accumulate, int64_t Bsz, int64_t L,
                int64_t D, int64_t N, int act, int dtype, void* ws, size_t ws_bytes,
                pgf_stream_t stream);

/* Saved scan states: pgf_ssm_fwd_save is pgf_ssm_fwd that also writes into `saved`
 * (pgf_ssm_saved_size bytes) the boundary state of every chunk and the state at the start of every
 * 8-token sub-chunk; pgf_ssm_bwd_saved is pgf_ssm_bwd for the same (u, parameters, h_init) that
 * reads them instead of recomputing its forward passes.  This is the reference's pgf_backward
 * recompute (pgf_mamba_block.py:157-178) feeding its block loop (:211-234) without a second scan.
 * The buffer holds (L/8 + L/Tc) * Bsz * D * N floats: O(L/8) states, not the (L, D, N) trajectory. */
size_t pgf_ssm_saved_size(int64_t Bsz, int64_t L, int64_t D, int64_t N);
/* The PGF boundary states alone, handed from the forward pass to the block's backward: fwd_states
 * is pgf_ssm_fwd that also writes every chunk's start state (and the end state) into `states`
 * (pgf_ssm_states_size bytes, the boundary states the reference recomputes at
 * pgf_mamba_block.py:157-175); fwd_save_states, given those states, produces the same y and
 * saved buffer as pgf_ssm_fwd_save in one pass over the sequence (no zero-start pass, compose or
 * correction). */
size_t pgf_ssm_states_size(int64_t Bsz, int64_t L, int64_t D, int64_t N);
int pgf_ssm_fwd_states(const void* u, const float* W_cat, const float* b_cat, const float* A_log, const float* Dp,
                       const float* scale, const float* h_init, void* y, float* states, int64_t Bsz, int64_t L,
                       int64_t D, int64_t N, int act, int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
int pgf_ssm_fwd_save_states(const void* u, const float* W_cat, const float* b_cat, const float* A_log,
                            const float* Dp, const float* scale, const float* states, void* y, float* saved,
                            int64_t Bsz, int64_t L, int64_t D, int64_t N, int act, int dtype, void* ws,
                            size_t ws_bytes, pgf_stream_t stream);
int pgf_ssm_fwd_save(const void* u, const float* W_cat, const float* b_cat, const float* A_log,
                     const float* Dp, const float* scale, const float* h_init, void* y, float* saved,
                     int64_t Bsz, int64_t L, int64_t D, int64_t N, int act, int dtype, void* ws,
                     size_t ws_bytes, pgf_stream_t stream);
int pgf_ssm_bwd_saved(const void* u, const void* g, const float* W_cat, const float* b_cat,
                      const float* A_log, const float* Dp, const float* scale, const float* saved,
                      const float* dh_end, const float* dA_end, float* grad_W_cat, float* grad_b_cat,
                      float* grad_A_log, float* grad_Dp, float* grad_scale, void* grad_u,
                      float* dh_start, float* dA_start, int accumulate, int64_t Bsz, int64_t L,
                      int64_t D, int64_t N, int act, int dtype, void* ws, size_t ws_bytes,
                      pgf_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Segment summaries for a sequence sharded across GPUs.  No single-function counterpart in the
 * reference: they are the block hand-off of pgf_mamba_block.py:86-112 (forward, `curr_h`) and
 * :207-234 (backward, `delta_h_next` / `dA_next`) made composable, using that the recurrence is
 * affine.  Workspace: pgf_ssm_workspace(..., backward = 0 / 1).
 *
 * pgf_ssm_summary: state after the segment starting from h_init (NULL = zeros) -> h_final
 *   (Bsz, D, N), and sum_dt (Bsz, D) = sum over the segment of softplus(dt_in), so that the
 *   segment's total decay is exp(A_n * sum_dt).
 * pgf_ssm_bwd_summary: adjoint at the segment's first token for a zero carry at its end ->
 *   dh_start (Bsz, D, N), the first token's decay dA_start = exp(dt_first A) (Bsz, D, N), and
 *   sum_dt_excl (Bsz, D) = sum of dt over every token but the first.  h_init is only read when
 *   act != PGF_ACT_NONE (the output activation's derivative needs the states).
 * ------------------------------------------------------------------------------------------ */
int pgf_ssm_summary(const void* u, const float* W_cat, const float* b_cat, const float* A_log,
                    const float* h_init, float* h_final, float* sum_dt, int64_t Bsz, int64_t L,
                    int64_t D, int64_t N, int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
int pgf_ssm_bwd_summary(const void* u, const void* g, const float* W_cat, const float* b_cat,
                        const float* A_log, const float* scale, const float* h_init, float* dh_start,
                        float* dA_start, float* sum_dt_excl, int64_t Bsz, int64_t L, int64_t D,
                        int64_t N, int act, int dtype, void* ws, size_t ws_bytes,
                        pgf_stream_t stream);

/* Staged scan for sequence sharding: one caller workspace (pgf_ssm_workspace(.., backward)) is
   carried from begin to finish.  fwd_begin: projection and the zero-start chunk pass; writes the
   segment's summary from a zero start (h_seg: state after the segment, sum_dt) -- what the ranks
   exchange.  fwd_finish: the output from the state entering the segment (h_init).  Together they
   equal pgf_ssm_fwd without a second projection or chunk pass.  bwd_begin (after pgf_ssm_fwd_save
   with the segment's h_init): the reverse chunk pass and the segment's adjoint summary for a zero
   end carry (as pgf_ssm_bwd_summary); bwd_finish: every gradient for the given end carry
   (as pgf_ssm_bwd_saved).  The same u, g, weights and `saved` in both calls. */
int pgf_ssm_fwd_begin(const void* u, const float* W_cat, const float* b_cat, const float* A_log, float* h_seg,
                      float* sum_dt, int64_t Bsz, int64_t L, int64_t D, int64_t N, int dtype, void* ws,
                      size_t ws_bytes, pgf_stream_t stream);
int pgf_ssm_fwd_finish(const void* u, const float* W_cat, const float* b_cat, const float* A_log, const float* Dp,
                       const float* scale, const float* h_init, void* y, float* h_final, int64_t Bsz, int64_t L,
                       int64_t D, int64_t N, int act, int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
/* pgf_ssm_fwd_finish that also writes the segment's boundary states (pgf_ssm_states_size bytes, the
 * state entering the segment folded in) for pgf_ssm_fwd_save_states: a sequence-sharded backward
 * (pgf_mamba_block.py:157-175 per segment) then skips the zero-start pass and compose. */
int pgf_ssm_fwd_finish_states(const void* u, const float* W_cat, const float* b_cat, const float* A_log,
                              const float* Dp, const float* scale, const float* h_init, void* y, float* states,
                              int64_t Bsz, int64_t L, int64_t D, int64_t N, int act, int dtype, void* ws,
                              size_t ws_bytes, pgf_stream_t stream);
int pgf_ssm_bwd_begin(const void* u, const void* g, const float* W_cat, const float* b_cat, const float* A_log,
                      const float* scale, const float* h_init, const float* saved, float* dh_start,
                      float* dA_start, float* sum_dt_excl, int64_t Bsz, int64_t L, int64_t D, int64_t N, int act,
                      int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
int pgf_ssm_bwd_finish(const void* u, const void* g, const float* W_cat, const float* b_cat, const float* A_log,
                       const float* Dp, const float* scale, const float* h_init, const float* saved,
                       const float* dh_end, const float* dA_end, float* gW_cat, float* gb_cat, float* gA_log,
                       float* gDp, float* gscale, void* gu, float* dh_start, float* dA_start, int accumulate,
                       int64_t Bsz, int64_t L, int64_t D, int64_t N, int act, int dtype, void* ws,
                       size_t ws_bytes, pgf_stream_t stream);
/* The block hand-off of the reference (pgf_mamba_block.py:86-112 forward, :207-234 backward) across
 * the P ranks of a sharded sequence, from the ranks' segment summaries gathered into one buffer
 * (`stride` floats per rank, rank order).  A_log is (N,) (shared) or, with a_per_channel, (D, N).
 *   fwd: rank j's entry is [h_seg (Bsz,D,N) | sum_dt (Bsz,D)] (pgf_ssm_fwd_begin); h_in = the fold
 *        H <- exp(A sum_dt_j) H + h_seg_j over j < rank from H = 0: the state entering `rank`.
 *   bwd: rank j's entry is [dh_start | dA_start (Bsz,D,N each) | sum_dt_excl (Bsz,D)]
 *        (pgf_ssm_bwd_begin); from G = 0, aE = 1, for j = P-1 down to rank+1:
 *        G <- exp(A sum_dt_excl_j) aE G + dh_start_j, aE <- dA_start_j; then dh_end = G, dA_end = aE. */
int pgf_ssm_compose_ranks_fwd(const float* gathered, int64_t stride, int P, int rank, const float* A_log,
                              int a_per_channel, float* h_in, int64_t Bsz, int64_t D, int64_t N,
                              pgf_stream_t stream);
int pgf_ssm_compose_ranks_bwd(const float* gathered, int64_t stride, int P, int rank, const float* A_log,
                              int a_per_channel, float* dh_end, float* dA_end, int64_t Bsz, int64_t D, int64_t N,
                              pgf_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Mamba-standard mixer: the variant the benchmark configurations describe; the reference has no
 * code for it (its SSM, train_singlemamba_optimized.py:88-124, has no in/out projection, conv or
 * gate).  x (Bsz, L, d) -> out (Bsz, L, d):
 *   xz = x in_w^T (in_w: 2E x d); xi, z = xz[:, :E], xz[:, E:]
 *   u = SiLU(causal depthwise conv1d(xi; conv_w (E, K), conv_b (E)))
 *   [dt_low | B | C] = u x_w^T (x_w: R+2N x E); delta = softplus(dt_low dt_w^T + dt_b) (dt_w: E x R)
 *   h_t = exp(delta_t A) h_{t-1} + delta_t B_t u_t, A = -exp(A_log) (E x N)
 *   y = (C_t . h_t + Dp u_t) * SiLU(z);  out = y out_w^T (out_w: d x E)
 * The backward re-runs the forward (keeping 8-token scan checkpoints) and returns every
 * parameter gradient and grad x.  N must be 16, K <= 8.  Zero initial state and conv history.
 * ------------------------------------------------------------------------------------------ */
size_t pgf_mamba_mixer_workspace(int64_t Bsz, int64_t L, int64_t d, int64_t E, int64_t R, int64_t N,
                                 int64_t K, int dtype, int backward);
int pgf_mamba_mixer_fwd(const void* x, const float* in_w, const float* conv_w, const float* conv_b,
                        const float* x_w, const float* dt_w, const float* dt_b, const float* A_log,
                        const float* Dp, const float* out_w, void* out, int64_t Bsz, int64_t L,
                        int64_t d, int64_t E, int64_t R, int64_t N, int64_t K, int dtype, void* ws,
                        size_t ws_bytes, pgf_stream_t stream);
int pgf_mamba_mixer_bwd(const void* x, const void* g_out, const float* in_w, const float* conv_w,
                        const float* conv_b, const float* x_w, const float* dt_w, const float* dt_b,
                        const float* A_log, const float* Dp, const float* out_w, float* g_in_w,
                        float* g_conv_w, float* g_conv_b, float* g_x_w, float* g_dt_w, float* g_dt_b,
                        float* g_A_log, float* g_Dp, float* g_out_w, void* g_x, int accumulate,
                        int64_t Bsz, int64_t L, int64_t d, int64_t E, int64_t R, int64_t N, int64_t K,
                        int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);

/* The mixer forward kept for its backward (the PGF block backward runs the mixer forward once,
   for the output the later operators need, and then its backward): fwd_save writes the forward
   intermediates (xz, u, y, x_dbl, dt, chunk states, 8-token scan checkpoints) into `saved`
   (>= pgf_mamba_mixer_saved_size bytes); bwd_saved reads them instead of re-running the forward.
   Same inputs and weights in both calls; `saved` is not modified by bwd_saved. */
size_t pgf_mamba_mixer_saved_size(int64_t Bsz, int64_t L, int64_t d, int64_t E, int64_t R, int64_t N,
                                  int64_t K, int dtype);
/* The scan's boundary states handed from the block forward to its backward (as
 * pgf_ssm_fwd_states / pgf_ssm_fwd_save_states): fwd_states is pgf_mamba_mixer_fwd that also writes
 * them (pgf_mamba_mixer_states_size bytes); fwd_save_states is pgf_mamba_mixer_fwd_save given them,
 * without the scan's chunk pass and compose. */
size_t pgf_mamba_mixer_states_size(int64_t Bsz, int64_t L, int64_t d, int64_t E, int64_t R, int64_t N, int64_t K);
int pgf_mamba_mixer_fwd_states(const void* x, const float* in_w, const float* conv_w, const float* conv_b,
                               const float* x_w, const float* dt_w, const float* dt_b, const float* A_log,
                               const float* Dp, const float* out_w, void* out, float* states, int64_t Bsz, int64_t L,
                               int64_t d, int64_t E, int64_t R, int64_t N, int64_t K, int dtype, void* ws,
                               size_t ws_bytes, pgf_stream_t stream);
int pgf_mamba_mixer_fwd_save_states(const void* x, const float* in_w, const float* conv_w, const float* conv_b,
                                    const float* x_w, const float* dt_w, const float* dt_b, const float* A_log,
                                    const float* Dp, const float* out_w, const float* states, void* out, void* saved,
                                    size_t saved_bytes, int64_t Bsz, int64_t L, int64_t d, int64_t E, int64_t R,
                                    int64_t N, int64_t K, int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
int pgf_mamba_mixer_fwd_save(const void* x, const float* in_w, const float* conv_w, const float* conv_b,
                             const float* x_w, const float* dt_w, const float* dt_b, const float* A_log,
                             const float* Dp, const float* out_w, void* out, void* saved, size_t saved_bytes,
                             int64_t Bsz, int64_t L, int64_t d, int64_t E, int64_t R, int64_t N, int64_t K,
                             int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
int pgf_mamba_mixer_bwd_saved(const void* x, const void* g_out, const float* in_w, const float* conv_w,
                              const float* conv_b, const float* x_w, const float* dt_w, const float* dt_b,
                              const float* A_log, const float* Dp, const float* out_w, float* g_in_w,
                              float* g_conv_w, float* g_conv_b, float* g_x_w, float* g_dt_w, float* g_dt_b,
                              float* g_A_log, float* g_Dp, float* g_out_w, void* g_x, int accumulate,
                              const void* saved, size_t saved_bytes, int64_t Bsz, int64_t L, int64_t d,
                              int64_t E, int64_t R, int64_t N, int64_t K, int dtype, void* ws, size_t ws_bytes,
                              pgf_stream_t stream);
/* The mixer over one segment of a longer sequence: the reference's block hand-off
 * (pgf_mamba_block.py:86-112 forward, :207-234 backward) for this variant, whose causal conv1d also
 * reads the K-1 tokens before the segment.  Carries (all nullable; NULL = the sequence starts or
 * ends here):
 *   x_halo  (Bsz, K-1, d): the mixer inputs of the K-1 tokens before the segment (conv context);
 *   h_init / h_final (Bsz, E, N): scan state entering / leaving the segment;
 *   dh_end / dA_end (Bsz, E, N): adjoint at the token after the segment and that token's decay
 *     exp(delta A); dh_start / dA_start: the same at the segment's first token, for the segment before;
 *   g_x_halo (Bsz, K-1, d): gradient of x_halo, to be added to the previous segment's input gradient
 *     (grad W_in already includes the halo rows' part).
 * fwd_seg: one call; states_in (from an earlier fwd_seg's states_out on the same input) replaces
 *   the chunk pass and compose, saved (pgf_mamba_mixer_saved_size bytes) keeps the forward for bwd_seg.
 * Staged (sequence sharding, one workspace carried between the two calls of a pair):
 *   fwd_begin: projections, conv, chunk pass; the segment's summary from a zero state (h_seg, sum_dt
 *   (Bsz, E): sum of delta).  fwd_finish: output from h_init (states_out: its boundary states).
 *   bwd_begin (saved from a fwd_seg with the segment's h_init): the adjoint summary for a zero end
 *   carry (dh_start, dA_start, sum_dt_excl (Bsz, E): sum of delta over every token but the first).
 *   bwd_finish: every gradient for the carry (dh_end, dA_end). */
int pgf_mamba_mixer_fwd_seg(const void* x, const float* in_w, const float* conv_w, const float* conv_b,
                            const float* x_w, const float* dt_w, const float* dt_b, const float* A_log, const float* Dp,
                            const float* out_w, const void* x_halo, const float* h_init, const float* states_in,
                            void* out, float* h_final, float* states_out, void* saved, size_t saved_bytes,
                            int64_t Bsz, int64_t L, int64_t d, int64_t E, int64_t R, int64_t N, int64_t K, int dtype,
                            void* ws, size_t ws_bytes, pgf_stream_t stream);
int pgf_mamba_mixer_fwd_begin(const void* x, const float* in_w, const float* conv_w, const float* conv_b,
                              const float* x_w, const float* dt_w, const float* dt_b, const float* A_log,
                              const float* Dp, const float* out_w, const void* x_halo, float* h_seg, float* sum_dt,
                              int64_t Bsz, int64_t L, int64_t d, int64_t E, int64_t R, int64_t N, int64_t K,
                              int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
int pgf_mamba_mixer_fwd_finish(const void* x, const float* in_w, const float* conv_w, const float* conv_b,
                               const float* x_w, const float* dt_w, const float* dt_b, const float* A_log,
                               const float* Dp, const float* out_w, const void* x_halo, const float* h_init, void* out,
                               float* states_out, int64_t Bsz, int64_t L, int64_t d, int64_t E, int64_t R, int64_t N,
                               int64_t K, int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
int pgf_mamba_mixer_bwd_seg(const void* x, const void* g_out, const float* in_w, const float* conv_w,
                            const float* conv_b, const float* x_w, const float* dt_w, const float* dt_b,
                            const float* A_log, const float* Dp, const float* out_w, const void* x_halo,
                            const void* saved, size_t saved_bytes, const float* dh_end, const float* dA_end,
                            float* g_in_w, float* g_conv_w, float* g_conv_b, float* g_x_w, float* g_dt_w,
                            float* g_dt_b, float* g_A_log, float* g_Dp, float* g_out_w, void* g_x, void* g_x_halo,
                            float* dh_start, float* dA_start, int accumulate, int64_t Bsz, int64_t L, int64_t d,
                            int64_t E, int64_t R, int64_t N, int64_t K, int dtype, void* ws, size_t ws_bytes,
                            pgf_stream_t stream);
int pgf_mamba_mixer_bwd_begin(const void* x, const void* g_out, const float* in_w, const float* conv_w,
                              const float* conv_b, const float* x_w, const float* dt_w, const float* dt_b,
                              const float* A_log, const float* Dp, const float* out_w, const void* x_halo,
                              const void* saved, size_t saved_bytes, float* dh_start, float* dA_start,
                              float* sum_dt_excl, int64_t Bsz, int64_t L, int64_t d, int64_t E, int64_t R, int64_t N,
                              int64_t K, int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
int pgf_mamba_mixer_bwd_finish(const void* x, const void* g_out, const float* in_w, const float* conv_w,
                               const float* conv_b, const float* x_w, const float* dt_w, const float* dt_b,
                               const float* A_log, const float* Dp, const float* out_w, const void* x_halo,
                               const void* saved, size_t saved_bytes, const float* dh_end, const float* dA_end,
                               float* g_in_w, float* g_conv_w, float* g_conv_b, float* g_x_w, float* g_dt_w,
                               float* g_dt_b, float* g_A_log, float* g_Dp, float* g_out_w, void* g_x,
                               void* g_x_halo, int accumulate, int64_t Bsz, int64_t L, int64_t d, int64_t E,
                               int64_t R, int64_t N, int64_t K, int dtype, void* ws, size_t ws_bytes,
                               pgf_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * The optimizer step after the PGF backward: the reference calls torch.optim.AdamW(lr=1e-3,
 * weight_decay=0.01, betas (0.9, 0.999), eps 1e-8) on all parameters (train_wikitext_rebuttal.py:
 * 77,148).  Here over ONE flat float32 buffer of n parameters with its flat gradient and moments.
 * pgf_adamw_step: that optimizer's update per element (decoupled weight decay, bias-corrected
 * moments) with the step count t read from and incremented in *step (device float, so a captured
 * step replays with the right t); grad_scale (device float or NULL) multiplies every gradient (the
 * clip factor).  All buffers 16-byte aligned.
 * pgf_grad_norm: the global L2 norm of the flat gradient (torch.nn.utils.clip_grad_norm_ over all
 * parameters) into *norm, and, when clip is non-NULL, the factor min(1, max_norm / (norm + 1e-6))
 * into *clip; deterministic (fixed block partition, partials summed in block order). */
int pgf_adamw_step(float* param, const float* grad, float* exp_avg, float* exp_avg_sq, int64_t n, float lr,
                   float beta1, float beta2, float eps, float weight_decay, float* step, const float* grad_scale,
                   pgf_stream_t stream);
/* pgf_adamw_step_multi: the same update with the gradients left in their own tensors: tensor i
 * (grads[i], NULL = zero gradient) covers the flat elements [offsets[i], offsets[i] + sizes[i]);
 * offsets multiples of 4.  grads / offsets / sizes are host arrays, read during the call (the
 * chunk table travels in the launch parameters, so a captured launch keeps it).
 * pgf_gather_multi: copies those tensors into the flat buffer dst (for a flat gradient that is then
 * all-reduced or clipped). */
int pgf_adamw_step_multi(float* param, float* exp_avg, float* exp_avg_sq, int64_t n, const float* const* grads,
                         const int64_t* offsets, const int64_t* sizes, int count, float lr, float beta1,
                         float beta2, float eps, float weight_decay, float* step, const float* grad_scale,
                         pgf_stream_t stream);
int pgf_gather_multi(float* dst, int64_t n, const float* const* srcs, const int64_t* offsets, const int64_t* sizes,
                     int count, pgf_stream_t stream);
size_t pgf_grad_norm_workspace(int64_t n);
int pgf_grad_norm(const float* grad, int64_t n, float* norm, float max_norm, float* clip, void* ws,
                  size_t ws_bytes, pgf_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Forward-mode (JVP) operators: directional derivatives computed alongside the forward, the
 * reference's forward-mode PGF path.
 * pgf_rmsnorm_jvp replaces RMSNorm.pgf_jvp (pgf_rmsnorm.py:54-72, 119-155): y and its derivative
 *   along (x_dot, weight_dot).
 * pgf_ffn_jvp replaces pgf_ffn_jvp (pgf_ffn.py:120-180): y = act(x W1^T + b1) W2^T + b2 and its
 *   derivative along every input's tangent (x_dot, W1_dot, b1_dot, W2_dot, b2_dot); rows are
 *   processed in tiles bounded by the workspace.
 * pgf_frechet_jvp replaces the scan of FrechetMambaOperator.pgf_forward (pgf_mamba.py:69-139) over
 *   a whole (L, D) sequence: W_cat = [dt_proj.weight; B_proj.weight; C_proj.weight] (D+2N, D),
 *   b_cat likewise, scale = redshift_scale (device scalar), h0 / h0_dot (D, N) the initial state
 *   and its tangent (NULL = zero; the operator's init_estimator produces them), outputs y, y_dot
 *   (L, D) and, when non-NULL, the end state and its tangent.  float32; N must be 16.
 * ------------------------------------------------------------------------------------------ */
int pgf_rmsnorm_jvp(const void* x, const void* x_dot, const float* weight, const float* weight_dot, void* y,
                    void* y_dot, int64_t rows, int64_t dim, float eps, int dtype, pgf_stream_t stream);
size_t pgf_ffn_jvp_workspace(int64_t rows, int64_t d_in, int64_t d_hidden, int64_t d_out, int dtype);
int pgf_ffn_jvp(const void* x, const void* x_dot, const float* W1, const float* W1_dot, const float* b1,
                const float* b1_dot, const float* W2, const float* W2_dot, const float* b2, const float* b2_dot,
                void* y, void* y_dot, int64_t rows, int64_t d_in, int64_t d_hidden, int64_t d_out, int activation,
                int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
size_t pgf_frechet_jvp_workspace(int64_t L, int64_t D, int64_t N);
/* State Hessian-vector product: replaces SingleLayerMambaPGF.compute_state_hvp
 * (train_singlemamba_optimized.py:563-685, HVP branch :249-275) for the MSE loss against target
 * (B, L, D): out (L, B, D, N) = the trajectory of d^2 Loss / dh^2 . v_h with v_h (B, D, N) the
 * direction on the initial state.  Same weights as pgf_ssm_fwd; float32; N must be 16. */
size_t pgf_ssm_state_hvp_workspace(int64_t Bsz, int64_t L, int64_t D, int64_t N, int act);
int pgf_ssm_state_hvp(const float* u, const float* target, const float* W_cat, const float* b_cat,
                      const float* A_log, const float* Dp, const float* scale, const float* v_h, float* out,
                      int64_t Bsz, int64_t L, int64_t D, int64_t N, int act, void* ws, size_t ws_bytes,
                      pgf_stream_t stream);
int pgf_frechet_jvp(const float* u, const float* u_dot, const float* W_cat, const float* b_cat, const float* A_log,
                    const float* Dp, const float* scale, const float* h0, const float* h0_dot, float* y,
                    float* y_dot, float* h_end, float* h_end_dot, int64_t L, int64_t D, int64_t N, void* ws,
                    size_t ws_bytes, pgf_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PGF_H_ */
