// FFN and LM-head operators composed from the dense-product engine
// (pgf_ffn.py:34-117, 183-307; pgf_lm_head.py:14-130; CE of test_multi_layer_grads.py:74-86).
//
// Rows (tokens) are processed in tiles whose scratch is bounded by the tile, not by the number
// of rows, which is the block-streaming of the reference on the GPU.  In bf16 mode the fp32
// master weights are converted once per call into bf16 operand copies in the workspace.
#include "gemm.cuh"

#include <math.h>
#include <stdlib.h>

namespace pgf {

static const int64_t kTileBytes = int64_t(128) << 20;  // scratch budget for one row tile
// The FFN's budget is larger: each row tile of the backward pays a split-K reduction and two column
// sums of its own, so a 65536-token sequence at d_hidden 1024 in bf16 runs as one tile.
static const int64_t kFfnTileBytes = int64_t(256) << 20;

static int64_t ffn_tile_rows(int64_t rows, int64_t d_hidden, int backward, int dtype) {
  // hidden activations (and the pre-activation in backward) of one tile, in the activation dtype
  int64_t per_row = d_hidden * (dtype ? 2 : 4) * (backward ? 2 : 1);
  int64_t t = kFfnTileBytes / (per_row > 0 ? per_row : 1);
  t = (t / 128) * 128;
  if (t < 128) t = 128;
  return rows < t ? rows : t;
}

struct FfnWs {
  void* h;      // tile hidden activations (dtype)
  void* z;      // tile pre-activation (backward): bf16 in bf16 runs (act' is evaluated at bf16 precision)
  __nv_bfloat16 *W1b, *W2b;  // bf16 operand copies
  void* cs;     // colsum scratch
  size_t cs_bytes;
  void* split;  // split-K partials of the weight gradients
  size_t split_bytes;
};

static size_t ffn_split_bytes(int64_t tr, int64_t d_in, int64_t d_h, int64_t d_out) {
  const size_t a = gemm_split_ws(d_out, d_h, tr), b = gemm_split_ws(d_h, d_in, tr);
  return a > b ? a : b;
}

static size_t ffn_ws_bytes(int64_t rows, int64_t d_in, int64_t d_h, int64_t d_out, int dtype, int backward) {
  int64_t tr = ffn_tile_rows(rows < 1 ? 1 : rows, d_h, backward, dtype);
  size_t es = dtype ? 2 : 4;
  size_t b = Workspace::round(size_t(tr) * d_h * es);
  if (backward) b += Workspace::round(size_t(tr) * d_h * es);
  if (dtype) b += Workspace::round(size_t(d_h) * d_in * 2) + Workspace::round(size_t(d_out) * d_h * 2);
  if (backward) {
    size_t c1 = colsum_ws(tr, d_h), c2 = colsum_ws(tr, d_out);
    b += Workspace::round(c1 > c2 ? c1 : c2);
    b += Workspace::round(ffn_split_bytes(tr, d_in, d_h, d_out));
  }
  return b + 1024;
}

static int ffn_carve(Workspace& W, FfnWs& f, int64_t rows, int64_t d_in, int64_t d_h, int64_t d_out,
                     int dtype, int backward) {
  int64_t tr = ffn_tile_rows(rows, d_h, backward, dtype);
  size_t es = dtype ? 2 : 4;
  f.h = W.take<char>(size_t(tr) * d_h * es);
  f.z = backward ? W.take<char>(size_t(tr) * d_h * es) : nullptr;
  f.W1b = dtype ? W.take<__nv_bfloat16>(size_t(d_h) * d_in) : nullptr;
  f.W2b = dtype ? W.take<__nv_bfloat16>(size_t(d_out) * d_h) : nullptr;
  if (backward) {
    size_t c1 = colsum_ws(tr, d_h), c2 = colsum_ws(tr, d_out);
    f.cs_bytes = c1 > c2 ? c1 : c2;
    f.cs = W.take<char>(f.cs_bytes);
    f.split_bytes = ffn_split_bytes(tr, d_in, d_h, d_out);
    f.split = f.split_bytes ? W.take<char>(f.split_bytes) : nullptr;
  } else {
    f.cs = nullptr;
    f.cs_bytes = 0;
    f.split = nullptr;
    f.split_bytes = 0;
  }
  if (!f.h || (backward && (!f.z || !f.cs || (f.split_bytes && !f.split))) || (dtype && (!f.W1b || !f.W2b))) {
    set_error("ffn: workspace too small (%zu)", W.cap);
    return PGF_ERR_WORKSPACE;
  }
  return PGF_OK;
}

static int act_epi(int activation, int backward) {
  if (activation == PGF_ACT_GELU) return backward ? PGF_EPI_DGELU : PGF_EPI_GELU;
  return backward ? PGF_EPI_DRELU : PGF_EPI_RELU;
}

static Gemm mk(int64_t M, int64_t N, int64_t K, const void* A, int abf, int64_t lda, int at,
               const void* B, int bbf, int64_t ldb, int bt, void* D, int dbf, int64_t ldd) {
  return gemm_make(M, N, K, A, abf, lda, at, B, bbf, ldb, bt, D, dbf, ldd);
}

}  // namespace pgf

using namespace pgf;

extern "C" size_t pgf_ffn_workspace(int64_t rows, int64_t d_in, int64_t d_hidden, int64_t d_out,
                                    int dtype, int backward) {
  return ffn_ws_bytes(rows, d_in, d_hidden, d_out, dtype, backward);
}

namespace pgf {
static int ffn_fwd_impl(const void* x, const float* W1, const float* b1, const float* W2, const float* b2,
                        const void* res, void* y, int64_t rows, int64_t d_in, int64_t d_hidden, int64_t d_out,
                        int activation, int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream);
}

extern "C" int pgf_ffn_fwd(const void* x, const float* W1, const float* b1, const float* W2,
                           const float* b2, void* y, int64_t rows, int64_t d_in, int64_t d_hidden,
                           int64_t d_out, int activation, int dtype, void* ws, size_t ws_bytes,
                           pgf_stream_t stream) {
  return ffn_fwd_impl(x, W1, b1, W2, b2, nullptr, y, rows, d_in, d_hidden, d_out, activation, dtype, ws, ws_bytes,
                      stream);
}

extern "C" int pgf_ffn_fwd_res(const void* x, const float* W1, const float* b1, const float* W2,
                               const float* b2, const void* res, void* y, int64_t rows, int64_t d_in,
                               int64_t d_hidden, int64_t d_out, int activation, int dtype, void* ws,
                               size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(res, "ffn_fwd_res: null residual");
  return ffn_fwd_impl(x, W1, b1, W2, b2, res, y, rows, d_in, d_hidden, d_out, activation, dtype, ws, ws_bytes,
                      stream);
}

namespace pgf {
static int ffn_fwd_impl(const void* x, const float* W1, const float* b1, const float* W2, const float* b2,
                        const void* res, void* y, int64_t rows, int64_t d_in, int64_t d_hidden, int64_t d_out,
                        int activation, int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(x && W1 && b1 && W2 && b2 && y, "ffn_fwd: null pointer");
  PGF_CHECK_ARG(activation == PGF_ACT_GELU || activation == PGF_ACT_RELU, "ffn_fwd: bad activation");
  PGF_CHECK_ARG(dtype == 0 || dtype == 1, "ffn_fwd: bad dtype");
  if (rows == 0) return PGF_OK;
  cudaStream_t s = as_stream(stream);
  Workspace W(ws, ws_bytes);
  FfnWs f;
  PGF_TRY(ffn_carve(W, f, rows, d_in, d_hidden, d_out, dtype, 0));
  const void* w1 = W1;
  const void* w2 = W2;
  if (dtype) {
    PGF_TRY(to_bf16_multi(Bf16Casts{{W1, W2}, {f.W1b, f.W2b}, {d_hidden * d_in, d_out * d_hidden}, 2}, s));
    w1 = f.W1b;
    w2 = f.W2b;
  }
  const int64_t tr = ffn_tile_rows(rows, d_hidden, 0, dtype);
  const size_t es = dtype ? 2 : 4;
  for (int64_t r = 0; r < rows; r += tr) {
    const int64_t m = rows - r < tr ? rows - r : tr;
    const char* xt = static_cast<const char*>(x) + r * d_in * es;
    char* yt = static_cast<char*>(y) + r * d_out * es;
    Gemm g1 = mk(m, d_hidden, d_in, xt, dtype, d_in, 0, w1, dtype, d_in, 0, f.h, dtype, d_hidden);
    g1.epi.bias = b1;
    g1.epi.kind = act_epi(activation, 0);
    PGF_TRY(run_gemm(g1, s));
    Gemm g2 = mk(m, d_out, d_hidden, f.h, dtype, d_hidden, 0, w2, dtype, d_hidden, 0, yt, dtype, d_out);
    g2.epi.bias = b2;
    if (res) {
      // y = h W2^T + b2 + res, rounded once (the block's FFN output plus its skip connection)
      g2.epi.addend = static_cast<const char*>(res) + r * d_out * es;
      g2.epi.addend_dtype = dtype;
      g2.epi.ld_addend = d_out;
    }
    PGF_TRY(run_gemm(g2, s));
  }
  return PGF_OK;
}
}  // namespace pgf

// ---------------------------------------------------------------------------------------------
// Forward-mode derivative (pgf_ffn_jvp, pgf_ffn.py:120-180), per row tile of m rows:
//   [h_dot | h] (m x 2H): h = act(x W1^T + b1) (GELU epilogue, z kept as aux), and
//   h_dot = ([x_dot | x] [W1 | W1_dot]^T + b1_dot) act'(z) (act' epilogue at z): the two terms of
//   z_dot as one product over the concatenated depth;
//   y = h W2^T + b2;  y_dot = [h_dot | h] [W2 | W2_dot]^T + b2_dot.
// Four dense products; only x (into [x_dot | x]) and the weights are copied, both with strided
// 2-D copies.
// ---------------------------------------------------------------------------------------------
namespace pgf {
static int64_t ffn_jvp_tile_rows(int64_t rows, int64_t d_in, int64_t d_h) {
  const int64_t per_row = (2 * d_in + 3 * d_h) * 4;
  int64_t t = kTileBytes / (per_row > 0 ? per_row : 1);
  t = (t / 128) * 128;
  if (t < 128) t = 128;
  return rows < t ? rows : t;
}
static size_t ffn_jvp_ws_bytes(int64_t rows, int64_t d_in, int64_t d_h, int64_t d_out, int dtype) {
  const int64_t tr = ffn_jvp_tile_rows(rows < 1 ? 1 : rows, d_in, d_h);
  const size_t es = dtype ? 2 : 4;
  size_t b = Workspace::round(size_t(d_h) * 2 * d_in * es) + Workspace::round(size_t(d_out) * 2 * d_h * es);
  if (dtype) {
    const size_t t1 = size_t(d_h) * d_in, t2 = size_t(d_out) * d_h;
    b += Workspace::round((t1 > t2 ? t1 : t2) * 2);
  }
  b += Workspace::round(size_t(tr) * 2 * d_in * es) + Workspace::round(size_t(tr) * d_h * es) +
       Workspace::round(size_t(tr) * 2 * d_h * es);
  return b + 1024;
}
// dst[:, off : off + cols] (pitch dpitch elements) = src (rows x cols float32), in dtype
static int copy_cols(void* dst, int64_t dpitch, int64_t off, const float* src, int64_t rows, int64_t cols, int dtype,
                     __nv_bfloat16* tmp, cudaStream_t s) {
  const size_t es = dtype ? 2 : 4;
  const void* from = src;
  if (dtype) {
    PGF_TRY(to_bf16(src, tmp, rows * cols, s));
    from = tmp;
  }
  PGF_CUDA(cudaMemcpy2DAsync(static_cast<char*>(dst) + off * es, dpitch * es, from, cols * es, cols * es, rows,
                             cudaMemcpyDeviceToDevice, s));
  return PGF_OK;
}
}  // namespace pgf

extern "C" size_t pgf_ffn_jvp_workspace(int64_t rows, int64_t d_in, int64_t d_hidden, int64_t d_out, int dtype) {
  return ffn_jvp_ws_bytes(rows, d_in, d_hidden, d_out, dtype);
}

extern "C" int pgf_ffn_jvp(const void* x, const void* x_dot, const float* W1, const float* W1_dot, const float* b1,
                           const float* b1_dot, const float* W2, const float* W2_dot, const float* b2,
                           const float* b2_dot, void* y, void* y_dot, int64_t rows, int64_t d_in, int64_t d_h,
                           int64_t d_out, int activation, int dtype, void* ws, size_t ws_bytes,
                           pgf_stream_t stream) {
  PGF_CHECK_ARG(x && x_dot && W1 && W1_dot && b1 && b1_dot && W2 && W2_dot && b2 && b2_dot && y && y_dot,
                "ffn_jvp: null pointer");
  PGF_CHECK_ARG(activation == PGF_ACT_GELU || activation == PGF_ACT_RELU, "ffn_jvp: bad activation");
  PGF_CHECK_ARG(dtype == 0 || dtype == 1, "ffn_jvp: bad dtype");
  PGF_CHECK_ARG(rows >= 0 && d_in > 0 && d_h > 0 && d_out > 0, "ffn_jvp: bad shape");
  if (rows == 0) return PGF_OK;
  cudaStream_t s = as_stream(stream);
  const size_t es = dtype ? 2 : 4;
  const int64_t tr = ffn_jvp_tile_rows(rows, d_in, d_h);
  Workspace W(ws, ws_bytes);
  char* B1 = W.take<char>(size_t(d_h) * 2 * d_in * es);   // [W1 | W1_dot]
  char* B2 = W.take<char>(size_t(d_out) * 2 * d_h * es);  // [W2 | W2_dot]
  __nv_bfloat16* tmp = nullptr;
  if (dtype) {
    const size_t t1 = size_t(d_h) * d_in, t2 = size_t(d_out) * d_h;
    tmp = W.take<__nv_bfloat16>(t1 > t2 ? t1 : t2);
  }
  char* A1 = W.take<char>(size_t(tr) * 2 * d_in * es);    // [x_dot | x] of a tile
  char* Z = W.take<char>(size_t(tr) * d_h * es);          // pre-activation of a tile
  char* HH = W.take<char>(size_t(tr) * 2 * d_h * es);     // [h_dot | h] of a tile
  if (!B1 || !B2 || (dtype && !tmp) || !A1 || !Z || !HH) {
    set_error("ffn_jvp: workspace too small (%zu)", ws_bytes);
    return PGF_ERR_WORKSPACE;
  }
  PGF_TRY(copy_cols(B1, 2 * d_in, 0, W1, d_h, d_in, dtype, tmp, s));
  PGF_TRY(copy_cols(B1, 2 * d_in, d_in, W1_dot, d_h, d_in, dtype, tmp, s));
  PGF_TRY(copy_cols(B2, 2 * d_h, 0, W2, d_out, d_h, dtype, tmp, s));
  PGF_TRY(copy_cols(B2, 2 * d_h, d_h, W2_dot, d_out, d_h, dtype, tmp, s));
  for (int64_t r = 0; r < rows; r += tr) {
    const int64_t m = rows - r < tr ? rows - r : tr;
    const char* xt = static_cast<const char*>(x) + r * d_in * es;
    const char* xdt = static_cast<const char*>(x_dot) + r * d_in * es;
    PGF_CUDA(cudaMemcpy2DAsync(A1, 2 * d_in * es, xdt, d_in * es, d_in * es, m, cudaMemcpyDeviceToDevice, s));
    PGF_CUDA(cudaMemcpy2DAsync(A1 + d_in * es, 2 * d_in * es, xt, d_in * es, d_in * es, m, cudaMemcpyDeviceToDevice,
                               s));
    // h = act(x W1^T + b1) into the right half of HH, z kept
    Gemm g1 = mk(m, d_h, d_in, A1 + d_in * es, dtype, 2 * d_in, 0, B1, dtype, 2 * d_in, 0, HH + d_h * es, dtype,
                 2 * d_h);
    g1.epi.bias = b1;
    g1.epi.kind = act_epi(activation, 0);
    g1.epi.aux_out = Z;
    g1.epi.aux_out_dtype = dtype;
    g1.epi.ld_aux_out = d_h;
    PGF_TRY(run_gemm(g1, s));
    // h_dot = ([x_dot | x] [W1 | W1_dot]^T + b1_dot) act'(z) into the left half
    Gemm g2 = mk(m, d_h, 2 * d_in, A1, dtype, 2 * d_in, 0, B1, dtype, 2 * d_in, 0, HH, dtype, 2 * d_h);
    g2.epi.bias = b1_dot;
    g2.epi.kind = act_epi(activation, 1);
    g2.epi.aux = Z;
    g2.epi.aux_dtype = dtype;
    g2.epi.ld_aux = d_h;
    PGF_TRY(run_gemm(g2, s));
    // y = h W2^T + b2
    Gemm g3 = mk(m, d_out, d_h, HH + d_h * es, dtype, 2 * d_h, 0, B2, dtype, 2 * d_h, 0,
                 static_cast<char*>(y) + r * d_out * es, dtype, d_out);
    g3.epi.bias = b2;
    PGF_TRY(run_gemm(g3, s));
    // y_dot = [h_dot | h] [W2 | W2_dot]^T + b2_dot
    Gemm g4 = mk(m, d_out, 2 * d_h, HH, dtype, 2 * d_h, 0, B2, dtype, 2 * d_h, 0,
                 static_cast<char*>(y_dot) + r * d_out * es, dtype, d_out);
    g4.epi.bias = b2_dot;
    PGF_TRY(run_gemm(g4, s));
  }
  return PGF_OK;
}

extern "C" int pgf_ffn_bwd(const void* x, const void* g, const float* W1, const float* b1,
                           const float* W2, float* gW1, float* gb1, float* gW2, float* gb2,
                           void* gx, int accumulate, int64_t rows, int64_t d_in, int64_t d_h,
                           int64_t d_out, int activation, int dtype, void* ws, size_t ws_bytes,
                           pgf_stream_t stream) {
  PGF_CHECK_ARG(x && g && W1 && b1 && W2 && gW1 && gb1 && gW2 && gb2, "ffn_bwd: null pointer");
  PGF_CHECK_ARG(activation == PGF_ACT_GELU || activation == PGF_ACT_RELU, "ffn_bwd: bad activation");
  PGF_CHECK_ARG(dtype == 0 || dtype == 1, "ffn_bwd: bad dtype");
  cudaStream_t s = as_stream(stream);
  if (rows == 0) {
    if (!accumulate) {
      PGF_CUDA(cudaMemsetAsync(gW1, 0, d_h * d_in * 4, s));
      PGF_CUDA(cudaMemsetAsync(gb1, 0, d_h * 4, s));
      PGF_CUDA(cudaMemsetAsync(gW2, 0, d_out * d_h * 4, s));
      PGF_CUDA(cudaMemsetAsync(gb2, 0, d_out * 4, s));
    }
    return PGF_OK;
  }
  Workspace W(ws, ws_bytes);
  FfnWs f;
  PGF_TRY(ffn_carve(W, f, rows, d_in, d_h, d_out, dtype, 1));
  const void* w1 = W1;
  const void* w2 = W2;
  int wbf = 0;
  if (dtype) {
    PGF_TRY(to_bf16_multi(Bf16Casts{{W1, W2}, {f.W1b, f.W2b}, {d_h * d_in, d_out * d_h}, 2}, s));
    w1 = f.W1b;
    w2 = f.W2b;
    wbf = 1;
  }
  const int64_t tr = ffn_tile_rows(rows, d_h, 1, dtype);
  const size_t es = dtype ? 2 : 4;
  for (int64_t r = 0; r < rows; r += tr) {
    const int64_t m = rows - r < tr ? rows - r : tr;
    const int acc = (r > 0) || accumulate;
    const char* xt = static_cast<const char*>(x) + r * d_in * es;
    const char* gt = static_cast<const char*>(g) + r * d_out * es;
    // bf16 on the tensor cores at shallow depths: h = act(x W1^T + b1) into f.h and
    // grad_z = (g W2) * act'(z) into f.z from one kernel, z kept in tensor memory.  Its 128-column
    // tiles pay off where the two epilogues, not the operand reads, bound the separate products
    // (measured: d_model 256 faster, d_model 1024 slower than the two products).
    bool dual = false;
    if (dtype && d_in + d_out <= 1024) {
      DualGemm dg;
      dg.M = m; dg.N = d_h; dg.K1 = d_in; dg.K2 = d_out;
      dg.A1 = xt; dg.lda1 = d_in; dg.B1 = w1; dg.ldb1 = d_in; dg.b1_trans = 0;
      dg.A2 = gt; dg.lda2 = d_out; dg.B2 = w2; dg.ldb2 = d_h; dg.b2_trans = 1;
      dg.bias = b1;
      dg.kind = act_epi(activation, 0);
      dg.H = f.h; dg.ldh = d_h;
      dg.DZ = f.z; dg.lddz = d_h;
      const int rc = run_gemm_tc_dual(dg, s);
      if (rc == PGF_OK) {
        dual = true;
      } else if (rc != PGF_ERR_UNSUPPORTED) {
        return rc;
      } else {
        clear_error();
      }
    }
    if (!dual) {
      // z = x W1^T + b1 and h = act(z), both in the activation dtype
      Gemm g1 = mk(m, d_h, d_in, xt, dtype, d_in, 0, w1, wbf, d_in, 0, f.h, dtype, d_h);
      g1.epi.bias = b1;
      g1.epi.kind = act_epi(activation, 0);
      g1.epi.aux_out = f.z;
      g1.epi.aux_out_dtype = dtype;
      g1.epi.ld_aux_out = d_h;
      PGF_TRY(run_gemm(g1, s));
    }
    // grad_W2 (+)= g^T h   (d_out x d_h, K = rows)
    Gemm g2 = mk(d_out, d_h, m, gt, dtype, d_out, 1, f.h, dtype, d_h, 1, gW2, 0, d_h);
    g2.epi.accumulate = acc;
    g2.ws = f.split; g2.ws_bytes = f.split_bytes;
    PGF_TRY(run_gemm(g2, s));
    PGF_TRY(colsum(gt, dtype, m, d_out, d_out, gb2, acc, f.cs, f.cs_bytes, s));
    void* gz = f.z;
    if (!dual) {
      // grad_z = (g W2) * act'(z), written over h (no longer needed)
      Gemm g3 = mk(m, d_h, d_out, gt, dtype, d_out, 0, w2, wbf, d_h, 1, f.h, dtype, d_h);
      g3.epi.kind = act_epi(activation, 1);
      g3.epi.aux = f.z;
      g3.epi.aux_dtype = dtype;
      g3.epi.ld_aux = d_h;
      PGF_TRY(run_gemm(g3, s));
      gz = f.h;
    }
    // grad_W1 (+)= grad_z^T x   (d_h x d_in, K = rows)
    Gemm g4 = mk(d_h, d_in, m, gz, dtype, d_h, 1, xt, dtype, d_in, 1, gW1, 0, d_in);
    g4.epi.accumulate = acc;
    g4.ws = f.split; g4.ws_bytes = f.split_bytes;
    PGF_TRY(run_gemm(g4, s));
    PGF_TRY(colsum(gz, dtype, m, d_h, d_h, gb1, acc, f.cs, f.cs_bytes, s));
    if (gx) {
      // grad_x = grad_z W1
      char* gxt = static_cast<char*>(gx) + r * d_in * es;
      Gemm g5 = mk(m, d_in, d_h, gz, dtype, d_h, 0, w1, wbf, d_in, 1, gxt, dtype, d_in);
      PGF_TRY(run_gemm(g5, s));
    }
  }
  return PGF_OK;
}

// ---------------------------------------------------------------------------
// LM head
// ---------------------------------------------------------------------------
extern "C" size_t pgf_lm_head_workspace(int64_t T, int64_t V, int64_t d, int dtype) {
  (void)T;
  return dtype ? Workspace::round(size_t(V) * d * 2) + 256 : 256;
}

extern "C" int pgf_lm_head_fwd(const void* h, const float* W, float* logits, int64_t T, int64_t V,
                               int64_t d, int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(h && W && logits, "lm_head_fwd: null pointer");
  cudaStream_t s = as_stream(stream);
  const void* w = W;
  if (dtype) {
    Workspace Wk(ws, ws_bytes);
    __nv_bfloat16* wb = Wk.take<__nv_bfloat16>(size_t(V) * d);
    if (!wb) { set_error("lm_head_fwd: workspace too small"); return PGF_ERR_WORKSPACE; }
    PGF_TRY(to_bf16(W, wb, V * d, s));
    w = wb;
  }
  Gemm g = mk(T, V, d, h, dtype, d, 0, w, dtype, d, 0, logits, 0, V);
  return run_gemm(g, s);
}

extern "C" int pgf_lm_head_bwd(const void* h, const float* g_logits, const float* W, float* grad_W,
                               void* grad_h, int accumulate, int64_t T, int64_t V, int64_t d,
                               int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(h && g_logits && W && grad_W, "lm_head_bwd: null pointer");
  (void)ws; (void)ws_bytes;
  cudaStream_t s = as_stream(stream);
  Gemm g1 = mk(V, d, T, g_logits, 0, V, 1, h, dtype, d, 1, grad_W, 0, d);
  g1.epi.accumulate = accumulate;
  PGF_TRY(run_gemm(g1, s));
  if (grad_h) {
    Gemm g2 = mk(T, d, V, g_logits, 0, V, 0, W, 0, d, 1, grad_h, dtype, d);
    PGF_TRY(run_gemm(g2, s));
  }
  return PGF_OK;
}

// ---------------------------------------------------------------------------
// LM head + cross entropy, tiled over (tokens x vocab)
// ---------------------------------------------------------------------------
namespace pgf {

constexpr int64_t CE_VT = 8192;  // vocab columns per tile

static int64_t ce_tile_rows(int64_t T) {
  int64_t t = kTileBytes / (CE_VT * 4);  // float32 logits tile
  t = (t / 128) * 128;
  if (t < 128) t = 128;
  return T < t ? T : t;
}

// Online log-sum-exp over one vocab tile: run_m/run_s hold the running max and sum of
// exp(logit - max) of each row; tgt_logit receives the target's logit when it lies in the tile.
__global__ void ce_tile_stats_kernel(const float* __restrict__ tile, int64_t rows, int64_t cols,
                                     int64_t ld, int64_t v0, const int64_t* __restrict__ targets,
                                     float* __restrict__ run_m, float* __restrict__ run_s,
                                     float* __restrict__ tgt_logit, int first) {
  const int lane = threadIdx.x & 31;
  const int64_t r = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float* row = tile + r * ld;
  float mx = -INFINITY;
  for (int64_t c = lane; c < cols; c += 32) mx = fmaxf(mx, row[c]);
  mx = warp_max(mx);
  float se = 0.f;
  for (int64_t c = lane; c < cols; c += 32) se += expf(row[c] - mx);
  se = warp_sum(se);
  if (lane == 0) {
    const int64_t tg = targets[r];
    if (tg >= v0 && tg < v0 + cols) tgt_logit[r] = row[tg - v0];
    if (first) {
      run_m[r] = mx;
      run_s[r] = se;
    } else {
      const float m0 = run_m[r];
      const float m1 = fmaxf(m0, mx);
      run_s[r] = run_s[r] * expf(m0 - m1) + se * expf(mx - m1);
      run_m[r] = m1;
    }
  }
}

__global__ void ce_finish_kernel(const float* __restrict__ run_m, const float* __restrict__ run_s,
                                 const float* __restrict__ tgt_logit, int64_t rows,
                                 float* __restrict__ loss_rows, float* __restrict__ lse) {
  const int64_t r = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const float l = run_m[r] + logf(run_s[r]);
  lse[r] = l;
  loss_rows[r] = l - tgt_logit[r];
}

// g = (exp(logit - lse) - onehot) * scale, in place (float32) and as a bf16 copy when asked.
__global__ void ce_grad_tile_kernel(float* __restrict__ tile, __nv_bfloat16* __restrict__ tile_bf,
                                    int64_t rows, int64_t cols, int64_t ld, int64_t v0,
                                    const int64_t* __restrict__ targets, const float* __restrict__ lse,
                                    float scale) {
  const int64_t r = blockIdx.y;
  const int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= rows || c >= cols) return;
  const int64_t o = r * ld + c;
  float p = expf(tile[o] - lse[r]);
  if (targets[r] == v0 + c) p -= 1.0f;
  p *= scale;
  tile[o] = p;
  if (tile_bf) tile_bf[o] = __float2bfloat16_rn(p);
}

struct CeWs {
  float* tile;
  __nv_bfloat16* tile_bf;
  __nv_bfloat16* Wb;
  float *run_m, *run_s, *tgt;
  float* gh32;  // float32 grad_h accumulator of a bf16 run
};

static size_t ce_ws_bytes(int64_t T, int64_t V, int64_t d, int dtype) {
  int64_t tr = ce_tile_rows(T < 1 ? 1 : T);
  size_t b = Workspace::round(size_t(tr) * CE_VT * 4);
  if (dtype) b += Workspace::round(size_t(tr) * CE_VT * 2) + Workspace::round(size_t(V) * d * 2);
  b += 3 * Workspace::round(size_t(tr) * 4);
  if (dtype) b += Workspace::round(size_t(tr) * d * 4);
  return b + 1024;
}

static int ce_carve(Workspace& W, CeWs& c, int64_t T, int64_t V, int64_t d, int dtype) {
  int64_t tr = ce_tile_rows(T);
  c.tile = W.take<float>(size_t(tr) * CE_VT);
  c.tile_bf = dtype ? W.take<__nv_bfloat16>(size_t(tr) * CE_VT) : nullptr;
  c.Wb = dtype ? W.take<__nv_bfloat16>(size_t(V) * d) : nullptr;
  c.run_m = W.take<float>(tr);
  c.run_s = W.take<float>(tr);
  c.tgt = W.take<float>(tr);
  c.gh32 = dtype ? W.take<float>(size_t(tr) * d) : nullptr;
  if ((dtype && !c.gh32) || !c.tile || !c.run_m || !c.run_s || !c.tgt || (dtype && (!c.tile_bf || !c.Wb))) {
    set_error("lm_head_ce: workspace too small");
    return PGF_ERR_WORKSPACE;
  }
  return PGF_OK;
}

// ---- tensor-core path (bf16): fused online-LSE forward, bf16 G written by the logits epilogue
constexpr int CE_NG = 16;                 // 128-column tiles per forward work unit (2048 vocab ids)
// Rows of G (bf16, rows x vocab) materialised at a time; PGF_CE_BWD_ROWS (a multiple of 128) tunes it.
static int64_t ce_bwd_rows() {
  static int64_t r = 0;
  if (!r) {
    const char* e = getenv("PGF_CE_BWD_ROWS");
    long long v = e ? atoll(e) : 0;
    r = (v >= 128) ? (v / 128) * 128 : 16384;
  }
  return r;
}

// partial (max, sum) pairs per row: two column halves per group of CE_NG tiles
static int64_t ce_ngroups(int64_t V) { return 2 * (((V + 127) / 128 + CE_NG - 1) / CE_NG); }
static int64_t ce_ldv(int64_t V) { return (V + 63) / 64 * 64; }

// Rows of the forward's partial (max, sum) pairs held at a time: the rows run in chunks of this many,
// so the workspace does not grow with T beyond it.
constexpr int64_t CE_FWD_ROWS = 65536;

static size_t ce_tc_ws_bytes(int64_t T, int64_t V, int64_t d) {
  const int64_t R = T < ce_bwd_rows() ? T : ce_bwd_rows();
  const int64_t Rf = T < CE_FWD_ROWS ? T : CE_FWD_ROWS;
  size_t b = Workspace::round(size_t(V) * d * 2);                  // W bf16
  b += 2 * Workspace::round(size_t(Rf) * ce_ngroups(V) * 4);       // part_m, part_s
  b += Workspace::round(size_t(Rf) * 4);                           // target logits
  b += Workspace::round(size_t(R < 1 ? 1 : R) * ce_ldv(V) * 2);    // G
  return b + 1024;
}

// lse = M + log(sum_g s_g exp(m_g - M)), loss = lse - target logit, groups in fixed order.
__global__ void ce_combine_kernel(const float* __restrict__ part_m, const float* __restrict__ part_s,
                                  const float* __restrict__ tgt, int64_t rows, int64_t ng,
                                  float* __restrict__ loss_rows, float* __restrict__ lse) {
  const int64_t r = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float M = -INFINITY;
  for (int64_t g = 0; g < ng; ++g) M = fmaxf(M, part_m[r * ng + g]);
  float S = 0.f;
  for (int64_t g = 0; g < ng; ++g) S += part_s[r * ng + g] * expf(part_m[r * ng + g] - M);
  const float l = M + logf(S);
  lse[r] = l;
  loss_rows[r] = l - tgt[r];
}

}  // namespace pgf

extern "C" size_t pgf_lm_head_ce_workspace(int64_t T, int64_t V, int64_t d, int dtype) {
  size_t a = ce_ws_bytes(T, V, d, dtype);
  if (dtype) {
    size_t b = ce_tc_ws_bytes(T, V, d);
    if (b > a) a = b;
  }
  return a;
}

namespace pgf {

static int ce_fwd_tc(const void* h, const float* W, const int64_t* targets, float* loss_rows, float* lse,
                     int64_t T, int64_t V, int64_t d, void* ws, size_t ws_bytes, cudaStream_t s) {
  Workspace Wk(ws, ws_bytes);
  __nv_bfloat16* Wb = Wk.take<__nv_bfloat16>(size_t(V) * d);
  const int64_t ng = ce_ngroups(V);
  const int64_t Rf = T < CE_FWD_ROWS ? T : CE_FWD_ROWS;
  float* pm = Wk.take<float>(size_t(Rf) * ng);
  float* ps = Wk.take<float>(size_t(Rf) * ng);
  float* tg = Wk.take<float>(size_t(Rf));
  if (!Wb || !pm || !ps || !tg) { set_error("lm_head_ce_fwd: workspace too small"); return PGF_ERR_WORKSPACE; }
  Gemm g = mk(Rf, V, d, h, 1, d, 0, Wb, 1, d, 0, nullptr, 0, 0);
  if (!tc_usable(g)) return PGF_ERR_UNSUPPORTED;
  PGF_TRY(to_bf16(W, Wb, V * d, s));
  for (int64_t r = 0; r < T; r += Rf) {
    const int64_t m = T - r < Rf ? T - r : Rf;
    Gemm gc = mk(m, V, d, static_cast<const __nv_bfloat16*>(h) + r * d, 1, d, 0, Wb, 1, d, 0, nullptr, 0, 0);
    // all-ones bytes = NaN: a row whose target lies outside [0, V) is never written and gets a NaN loss
    PGF_CUDA(cudaMemsetAsync(tg, 0xFF, size_t(m) * 4, s));
    int ngo = 0;
    PGF_TRY(tc_ce_fwd(gc, CE_NG, targets + r, pm, ps, tg, &ngo, s));
    ce_combine_kernel<<<ceil_div(m, 256), 256, 0, s>>>(pm, ps, tg, m, ngo, loss_rows + r, lse + r);
    PGF_LAUNCH_CHECK();
  }
  return PGF_OK;
}

static bool fused_ce_disabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("PGF_CE_UNFUSED");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

static int ce_bwd_tc(const void* h, const float* W, const int64_t* targets, const float* lse, float scale,
                     float* grad_W, void* grad_h, int accumulate, int64_t T, int64_t V, int64_t d,
                     void* ws, size_t ws_bytes, cudaStream_t s) {
  Workspace Wk(ws, ws_bytes);
  __nv_bfloat16* Wb = Wk.take<__nv_bfloat16>(size_t(V) * d);
  const int64_t ng = ce_ngroups(V);
  const int64_t Rf = T < CE_FWD_ROWS ? T : CE_FWD_ROWS;
  Wk.take<float>(size_t(Rf) * ng);  // keep the forward layout: the same workspace serves both
  Wk.take<float>(size_t(Rf) * ng);
  Wk.take<float>(size_t(Rf));
  const int64_t R = T < ce_bwd_rows() ? T : ce_bwd_rows();
  const int64_t ldv = ce_ldv(V);
  __nv_bfloat16* G = Wk.take<__nv_bfloat16>(size_t(R) * ldv);
  if (!Wb || !G) { set_error("lm_head_ce_bwd: workspace too small"); return PGF_ERR_WORKSPACE; }
  Gemm probe = mk(R, V, d, h, 1, d, 0, Wb, 1, d, 0, G, 1, ldv);
  if (!tc_usable(probe)) return PGF_ERR_UNSUPPORTED;
  PGF_TRY(to_bf16(W, Wb, V * d, s));
  // grad_h through the fused kernel (G written once, dh accumulated in TMEM) when it applies
  const bool fused = grad_h && !fused_ce_disabled() && ce_bwd_dh_usable(h, Wb, G, ldv, grad_h, d);
  for (int64_t r = 0; r < T; r += R) {
    const int64_t m = T - r < R ? T - r : R;
    const __nv_bfloat16* ht = static_cast<const __nv_bfloat16*>(h) + r * d;
    __nv_bfloat16* ght = grad_h ? static_cast<__nv_bfloat16*>(grad_h) + r * d : nullptr;
    if (fused) {
      PGF_TRY(ce_bwd_dh(ht, Wb, targets + r, lse + r, scale, G, ldv, ght, m, V, d, s));
    } else {
      Gemm g = mk(m, V, d, ht, 1, d, 0, Wb, 1, d, 0, G, 1, ldv);
      PGF_TRY(tc_ce_bwd(g, targets + r, lse + r, scale, G, ldv, s));
    }
    // grad_W (+)= G^T h_rows
    Gemm gw = mk(V, d, m, G, 1, ldv, 1, ht, 1, d, 1, grad_W, 0, d);
    gw.epi.accumulate = (r > 0) || accumulate;
    PGF_TRY(run_gemm(gw, s));
    if (ght && !fused) {
      // grad_h_rows = G W
      Gemm gh = mk(m, d, V, G, 1, ldv, 0, Wb, 1, d, 1, ght, 1, d);
      PGF_TRY(run_gemm(gh, s));
    }
  }
  return PGF_OK;
}

}  // namespace pgf

extern "C" int pgf_lm_head_ce_fwd(const void* h, const float* W, const int64_t* targets,
                                  float* loss_rows, float* lse, int64_t T, int64_t V, int64_t d,
                                  int dtype, void* ws, size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(h && W && targets && loss_rows && lse, "lm_head_ce_fwd: null pointer");
  PGF_CHECK_ARG(dtype == 0 || dtype == 1, "lm_head_ce_fwd: bad dtype");
  if (T == 0) return PGF_OK;
  cudaStream_t s = as_stream(stream);
  if (dtype) {
    const int rc = ce_fwd_tc(h, W, targets, loss_rows, lse, T, V, d, ws, ws_bytes, s);
    if (rc != PGF_ERR_UNSUPPORTED) return rc;
    clear_error();
  }
  Workspace Wk(ws, ws_bytes);
  CeWs c;
  PGF_TRY(ce_carve(Wk, c, T, V, d, dtype));
  const void* w = W;
  if (dtype) {
    PGF_TRY(to_bf16(W, c.Wb, V * d, s));
    w = c.Wb;
  }
  const int64_t tr = ce_tile_rows(T);
  const size_t es = dtype ? 2 : 4;
  for (int64_t r = 0; r < T; r += tr) {
    const int64_t m = T - r < tr ? T - r : tr;
    const char* ht = static_cast<const char*>(h) + r * d * es;
    PGF_CUDA(cudaMemsetAsync(c.tgt, 0xFF, size_t(m) * 4, s));  // NaN loss for a target outside [0, V)
    for (int64_t v0 = 0; v0 < V; v0 += CE_VT) {
      const int64_t nv = V - v0 < CE_VT ? V - v0 : CE_VT;
      const int64_t ldt = (nv + 63) / 64 * 64;  // 128-byte aligned tile pitch (TMA operand rule)
      const char* wt = static_cast<const char*>(w) + v0 * d * es;
      Gemm g = mk(m, nv, d, ht, dtype, d, 0, wt, dtype, d, 0, c.tile, 0, ldt);
      PGF_TRY(run_gemm(g, s));
      ce_tile_stats_kernel<<<ceil_div(m, 8), 256, 0, s>>>(c.tile, m, nv, ldt, v0, targets + r, c.run_m,
                                                         c.run_s, c.tgt, v0 == 0);
      PGF_LAUNCH_CHECK();
    }
    ce_finish_kernel<<<ceil_div(m, 256), 256, 0, s>>>(c.run_m, c.run_s, c.tgt, m, loss_rows + r, lse + r);
    PGF_LAUNCH_CHECK();
  }
  return PGF_OK;
}

extern "C" int pgf_lm_head_ce_bwd(const void* h, const float* W, const int64_t* targets,
                                  const float* lse, float grad_scale, float* grad_W, void* grad_h,
                                  int accumulate, int64_t T, int64_t V, int64_t d, int dtype,
                                  void* ws, size_t ws_bytes, pgf_stream_t stream) {
  PGF_CHECK_ARG(h && W && targets && lse && grad_W, "lm_head_ce_bwd: null pointer");
  PGF_CHECK_ARG(dtype == 0 || dtype == 1, "lm_head_ce_bwd: bad dtype");
  cudaStream_t s = as_stream(stream);
  if (T == 0) {
    if (!accumulate) PGF_CUDA(cudaMemsetAsync(grad_W, 0, size_t(V) * d * 4, s));
    return PGF_OK;
  }
  if (dtype) {
    const int rc = ce_bwd_tc(h, W, targets, lse, grad_scale, grad_W, grad_h, accumulate, T, V, d, ws,
                             ws_bytes, s);
    if (rc != PGF_ERR_UNSUPPORTED) return rc;
    clear_error();
  }
  Workspace Wk(ws, ws_bytes);
  CeWs c;
  PGF_TRY(ce_carve(Wk, c, T, V, d, dtype));
  const void* w = W;
  if (dtype) {
    PGF_TRY(to_bf16(W, c.Wb, V * d, s));
    w = c.Wb;
  }
  const int64_t tr = ce_tile_rows(T);
  const size_t es = dtype ? 2 : 4;
  for (int64_t r = 0; r < T; r += tr) {
    const int64_t m = T - r < tr ? T - r : tr;
    const char* ht = static_cast<const char*>(h) + r * d * es;
    char* ght = grad_h ? static_cast<char*>(grad_h) + r * d * es : nullptr;
    for (int64_t v0 = 0; v0 < V; v0 += CE_VT) {
      const int64_t nv = V - v0 < CE_VT ? V - v0 : CE_VT;
      const int64_t ldt = (nv + 63) / 64 * 64;
      const char* wt = static_cast<const char*>(w) + v0 * d * es;
      Gemm g = mk(m, nv, d, ht, dtype, d, 0, wt, dtype, d, 0, c.tile, 0, ldt);
      PGF_TRY(run_gemm(g, s));
      dim3 gg(ceil_div(nv, 256), unsigned(m));
      ce_grad_tile_kernel<<<gg, 256, 0, s>>>(c.tile, c.tile_bf, m, nv, ldt, v0, targets + r, lse + r,
                                              grad_scale);
      PGF_LAUNCH_CHECK();
      const void* gt = dtype ? (const void*)c.tile_bf : (const void*)c.tile;
      // grad_W[v0:v0+nv] (+)= G^T h_tile
      Gemm gw = mk(nv, d, m, gt, dtype, ldt, 1, ht, dtype, d, 1, grad_W + v0 * d, 0, d);
      gw.epi.accumulate = (r > 0) || accumulate;
      PGF_TRY(run_gemm(gw, s));
      if (ght) {
        // grad_h_tile (+)= G W_tile, summed over vocab tiles in float32
        float* acc32 = dtype ? c.gh32 : reinterpret_cast<float*>(ght);
        Gemm gh = mk(m, d, nv, gt, dtype, ldt, 0, wt, dtype, d, 1, acc32, 0, d);
        gh.epi.accumulate = v0 > 0;
        PGF_TRY(run_gemm(gh, s));
      }
    }
    if (ght && dtype) PGF_TRY(to_bf16(c.gh32, reinterpret_cast<__nv_bfloat16*>(ght), m * d, s));
  }
  return PGF_OK;
}
