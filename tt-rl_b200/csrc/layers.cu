// Linear and Conv2d forward/backward expressed as tcgen05 GEMMs with fused
// epilogues, plus the two non-GEMM pieces they need: the col2im gather
// that finishes the convolution input gradient, and the uint8 frame
// normalisation that feeds the first convolution.
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace ttrl {

static ttrl_operand dense(const float* p, int rows, int kdim, long long rs, long long ks) {
  ttrl_operand o;
  std::memset(&o, 0, sizeof(o));
  o.ptr = p;
  o.kind = TTRL_OPND_DENSE;
  o.rows = rows;
  o.kdim = kdim;
  o.rs = rs;
  o.ks = ks;
  return o;
}

static ttrl_operand conv_operand(const float* p, int kind, const ttrl_conv_geom& g) {
  ttrl_operand o;
  std::memset(&o, 0, sizeof(o));
  o.ptr = p;
  o.kind = kind;
  const int m = g.n * g.oh * g.ow;
  const int kk = g.kh * g.kw * g.c;
  o.rows = kind == TTRL_OPND_CONV_FPROP ? m : kk;
  o.kdim = kind == TTRL_OPND_CONV_FPROP ? kk : m;
  o.n = g.n;
  o.h = g.h;
  o.w = g.w;
  o.c = g.c;
  o.kh = g.kh;
  o.kw = g.kw;
  o.stride = g.stride;
  o.pad = g.pad;
  o.oh = g.oh;
  o.ow = g.ow;
  if (g.flags & TTRL_CONV_INPUT_EXACT) o.flags |= TTRL_OPND_EXACT_TF32;
  return o;
}

static ttrl_epilogue epi(float* out, long long ors, long long ocs) {
  ttrl_epilogue e;
  std::memset(&e, 0, sizeof(e));
  e.out = out;
  e.ors = ors;
  e.ocs = ocs;
  e.alpha = 1.f;
  return e;
}

static ttrl_gemm_desc make_desc(int m, int n, int k, int precision) {
  ttrl_gemm_desc d;
  std::memset(&d, 0, sizeof(d));
  d.m = m;
  d.n = n;
  d.k = k;
  d.precision = precision;
  return d;
}

static int check_conv(const ttrl_conv_geom* g) {
  if (g == nullptr) return set_error(TTRL_EINVAL, "conv: null geometry");
  if (g->n <= 0 || g->h <= 0 || g->w <= 0 || g->c <= 0 || g->cout <= 0 || g->kh <= 0 ||
      g->kw <= 0 || g->stride <= 0 || g->pad < 0)
    return set_error(TTRL_EINVAL, "conv: non-positive extent in geometry");
  const int sh = g->h + 2 * g->pad - g->kh, sw = g->w + 2 * g->pad - g->kw;
  if (sh < 0 || sw < 0 || sh % g->stride || sw % g->stride)
    return set_error(TTRL_EINVAL,
                     "conv: ragged or empty geometry (h=%d w=%d k=%dx%d s=%d p=%d); the input "
                     "gradient is only the exact adjoint for exactly divisible strides",
                     g->h, g->w, g->kh, g->kw, g->stride, g->pad);
  if (g->oh != sh / g->stride + 1 || g->ow != sw / g->stride + 1)
    return set_error(TTRL_EINVAL, "conv: oh/ow (%d,%d) disagree with the geometry (%d,%d)", g->oh,
                     g->ow, sh / g->stride + 1, sw / g->stride + 1);
  return TTRL_OK;
}

// ---------------------------------------------------------------- Linear

// Workspace bytes linear_fwd needs: the same orientation rule as below
// (output features as tile rows when the batch is narrower).
size_t linear_fwd_ws(int m, int k, int n, int precision) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  return gemm_workspace_bytes(m < 128 && n > m ? make_desc(n, m, k, precision)
                                               : make_desc(m, n, k, precision));
}

int linear_fwd(const float* x, const float* w, const float* b, float* y, int m, int k, int n,
               int relu, int precision, float* ws, size_t wsb, int* status, cudaStream_t st) {
  if (m <= 0 || n <= 0 || k <= 0) return set_error(TTRL_EINVAL, "linear_fwd: bad extents");
  ttrl_gemm_desc d;
  if (m < 128 && n > m) {
    // Rows of the tile are output features, columns are batch rows.
    d = make_desc(n, m, k, precision);
    d.a = dense(w, n, k, 1, n);
    d.b = dense(x, m, k, k, 1);
    d.ep = epi(y, 1, n);
    if (b) {
      d.ep.bias = b;
      d.ep.bias_mode = TTRL_BIAS_ROW;
    }
  } else {
    d = make_desc(m, n, k, precision);
    d.a = dense(x, m, k, k, 1);
    d.b = dense(w, n, k, 1, n);
    d.ep = epi(y, n, 1);
    if (b) {
      d.ep.bias = b;
      d.ep.bias_mode = TTRL_BIAS_COL;
    }
  }
  d.ep.relu = relu;
  return gemm_run_ws(d, 0, no_extra(), ws, wsb, status, st);
}

int linear_dgrad(const float* g, const float* w, const float* mask, float* dx, int m, int k,
                 int n, int accumulate, int precision, float* ws, size_t wsb, int* status,
                 cudaStream_t st) {
  if (m <= 0 || n <= 0 || k <= 0) return set_error(TTRL_EINVAL, "linear_dgrad: bad extents");
  ttrl_gemm_desc d;
  if (m < 128 && k > m) {
    d = make_desc(k, m, n, precision);
    d.a = dense(w, k, n, n, 1);
    d.b = dense(g, m, n, n, 1);
    d.ep = epi(dx, 1, k);
    if (mask) {
      d.ep.mask = mask;
      d.ep.mrs = 1;
      d.ep.mcs = k;
    }
  } else {
    d = make_desc(m, k, n, precision);
    d.a = dense(g, m, n, n, 1);
    d.b = dense(w, k, n, n, 1);
    d.ep = epi(dx, k, 1);
    if (mask) {
      d.ep.mask = mask;
      d.ep.mrs = k;
      d.ep.mcs = 1;
    }
  }
  d.ep.accumulate = accumulate;
  return gemm_run_ws(d, 0, no_extra(), ws, wsb, status, st);
}

// Workspace of linear_wgrad: [counters | GEMM split-K partials].
size_t linear_wgrad_ws(int m, int k, int n) {
  return gemm_workspace_bytes(make_desc(k + 1, n, m, TTRL_PREC_TF32X3));
}

int linear_wgrad(const float* x, const float* g, float* dw, float* db, int m, int k, int n,
                 int accumulate, int accumulate_db, int precision, float* ws, size_t wsb,
                 int* status, cudaStream_t st) {
  if (m <= 0 || n <= 0 || k <= 0) return set_error(TTRL_EINVAL, "linear_wgrad: bad extents");
  // db rides along as an extra row of ones appended to x^T: its row of D
  // is the column sums of g, in the same GEMM and its tile-order reduction.
  ttrl_gemm_desc d = make_desc(k + (db ? 1 : 0), n, m, precision);
  d.a = dense(x, k, m, 1, k);
  d.b = dense(g, n, m, 1, n);
  d.ep = epi(dw, n, 1);
  d.ep.accumulate = accumulate;
  EpiExtra ex = no_extra();
  if (db) {
    ex.row2 = k;
    ex.out2 = db;
    ex.cs2 = 1;
    ex.accumulate2 = accumulate_db;
  }
  return gemm_run_ws(d, db ? 1 : 0, ex, ws, wsb, status, st);
}

// ------------------------------------------------------------------ Conv

int conv_fprop(const float* x, const float* w, const float* b, float* y, const ttrl_conv_geom* g,
               float alpha, int relu, int precision, float* ws, size_t wsb, int* status,
               cudaStream_t st) {
  int rc = check_conv(g);
  if (rc) return rc;
  const int m = g->n * g->oh * g->ow;
  const int kk = g->kh * g->kw * g->c;
  ttrl_gemm_desc d = make_desc(m, g->cout, kk, precision);
  d.a = conv_operand(x, TTRL_OPND_CONV_FPROP, *g);
  d.b = dense(w, g->cout, kk, kk, 1);
  d.ep = epi(y, g->cout, 1);
  d.ep.alpha = alpha;
  if (b) {
    d.ep.bias = b;
    d.ep.bias_mode = TTRL_BIAS_COL;
  }
  d.ep.relu = relu;
  return gemm_run_ws(d, 0, no_extra(), ws, wsb, status, st);
}

// dx[n,iy,ix,c] = sum over the kernel taps that saw (iy,ix) of dxcol, in a
// fixed (ky, kx) order, then the relu mask of the layer below.
// dX from the im2col-shaped gradient dxcol[m][(ky, kx, c)]: each input
// pixel sums, over the kernel taps that saw it, the matching column of the
// output pixel's row. One thread owns 4 channels of one pixel (C % 4 == 0)
// or one channel; indices are 32-bit with multiply-shift division, and all
// tap loads are issued before the sum, which runs in (ky, kx) order.
struct Col2imArgs {
  const float* dxcol;
  const float* mask;
  float* dx;
  ttrl_conv_geom g;
  FastDiv f_cg, f_w, f_h, f_s;
  int cg;  // channel groups per pixel: C / 4 (vector) or C
  int vec;
  int accumulate;
  int total;  // pixels * cg
};

constexpr int kCol2imMaxTaps = 16;

template <bool VEC>
__global__ void __launch_bounds__(256) col2im_kernel(const __grid_constant__ Col2imArgs a) {
  pdl_trigger();
  pdl_wait();
  const ttrl_conv_geom g = a.g;
  const int kk = g.kh * g.kw * g.c;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < a.total;
       idx += gridDim.x * blockDim.x) {
    const int pix = fdiv(a.f_cg, idx);
    const int c = (idx - pix * a.cg) * (VEC ? 4 : 1);
    const int t = fdiv(a.f_w, pix);
    const int ix = pix - t * g.w;
    const int img = fdiv(a.f_h, t);
    const int iy = t - img * g.h;
    const int ty0 = iy + g.pad, tx0 = ix + g.pad;
    const int ky0 = ty0 - fdiv(a.f_s, ty0) * g.stride;  // first tap row that saw this pixel
    const int kx0 = tx0 - fdiv(a.f_s, tx0) * g.stride;
    const long long base = static_cast<long long>(pix) * g.c + c;
    float4 old = make_float4(0.f, 0.f, 0.f, 0.f), mk = make_float4(1.f, 1.f, 1.f, 1.f);
    if (VEC) {
      if (a.accumulate) old = *reinterpret_cast<const float4*>(a.dx + base);
      if (a.mask) mk = *reinterpret_cast<const float4*>(a.mask + base);
    } else {
      if (a.accumulate) old.x = a.dx[base];
      if (a.mask) mk.x = a.mask[base];
    }
    float4 v[kCol2imMaxTaps];
    int nt = 0;
#pragma unroll
    for (int q = 0; q < kCol2imMaxTaps; ++q) v[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    // Taps in (ky, kx) order; at most 16 (enforced on the host).
    for (int ky = ky0; ky < g.kh; ky += g.stride) {
      const int oy = fdiv(a.f_s, ty0 - ky);
      if (ty0 - ky < 0 || oy >= g.oh) continue;
      for (int kx = kx0; kx < g.kw; kx += g.stride) {
        const int ox = fdiv(a.f_s, tx0 - kx);
        if (tx0 - kx < 0 || ox >= g.ow) continue;
        const long long off =
            (static_cast<long long>(img * g.oh + oy) * g.ow + ox) * kk + (ky * g.kw + kx) * g.c + c;
#pragma unroll
        for (int q = 0; q < kCol2imMaxTaps; ++q) {
          if (q == nt) {
            if (VEC) {
              v[q] = *reinterpret_cast<const float4*>(a.dxcol + off);
            } else {
              v[q].x = a.dxcol[off];
            }
          }
        }
        ++nt;
      }
    }
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < kCol2imMaxTaps; ++q) {
      if (q < nt) {
        s.x += v[q].x;
        s.y += v[q].y;
        s.z += v[q].z;
        s.w += v[q].w;
      }
    }
    if (a.mask) {
      if (!(mk.x > 0.f)) s.x = 0.f;
      if (!(mk.y > 0.f)) s.y = 0.f;
      if (!(mk.z > 0.f)) s.z = 0.f;
      if (!(mk.w > 0.f)) s.w = 0.f;
    }
    if (a.accumulate) {
      s.x += old.x;
      s.y += old.y;
      s.z += old.z;
      s.w += old.w;
    }
    if (VEC) {
      *reinterpret_cast<float4*>(a.dx + base) = s;
    } else {
      a.dx[base] = s.x;
    }
  }
}

// ------------------------------------------- direct (sub-pixel) data gradient
//
// For a convolution with no padding, a stride s that divides the kernel k
// and an input covered exactly by the windows (h = (oh - 1) s + k), the data
// gradient splits by input-pixel parity q = (py, px) into s^2 stride-1
// correlations of dY with sub-kernels of extent kb = k / s:
//   dX[n, s i + py, s j + px, c]
//     = sum_{ty, tx < kb, co} dY[n, i - (kb-1) + ty, j - (kb-1) + tx, co]
//                              * W[co, s (kb-1-ty) + py, s (kb-1-tx) + px, c]
// for i < h / s, j < w / s (dY read as zero outside its extent). All s^2
// classes read the same dY windows, so the whole gradient is ONE implicit
// GEMM: A = the windows of dY (a stride-1 conv operand, padding kb - 1),
// B = the s^2 sub-kernels stacked into an (s^2 C) x (kb^2 Cout) matrix, and
// the epilogue scatters column q * C + c of row (n, i, j) to its pixel. No
// column buffer and no col2im pass.

static bool direct_dgrad_enabled() {
  static int on = [] {
    const char* e = std::getenv("TTRL_DIRECT_DGRAD");
    return e ? std::atoi(e) : 1;
  }();
  return on != 0;
}

static bool direct_dgrad_applies(const ttrl_conv_geom* g) {
  if (!direct_dgrad_enabled()) return false;
  const int s = g->stride, k = g->kh;
  return g->pad == 0 && g->kh == g->kw && k % s == 0 && g->h == (g->oh - 1) * s + k &&
         g->w == (g->ow - 1) * s + k;
}

static size_t dgrad_weights_bytes(const ttrl_conv_geom* g) {
  const size_t n = static_cast<size_t>(g->kh) * g->kw * g->c * g->cout;
  return (n * sizeof(float) + 255) & ~static_cast<size_t>(255);
}

static ttrl_conv_geom dgrad_window_geom(const ttrl_conv_geom* g) {
  const int kb = g->kh / g->stride;
  ttrl_conv_geom a;
  std::memset(&a, 0, sizeof(a));
  a.n = g->n;
  a.h = g->oh;
  a.w = g->ow;
  a.c = g->cout;
  a.cout = g->stride * g->stride * g->c;
  a.kh = a.kw = kb;
  a.stride = 1;
  a.pad = kb - 1;
  a.oh = g->h / g->stride;
  a.ow = g->w / g->stride;
  return a;
}

static ttrl_gemm_desc direct_dgrad_desc(const ttrl_conv_geom* g, int precision) {
  const ttrl_conv_geom a = dgrad_window_geom(g);
  const int kb = a.kh;
  return make_desc(a.n * a.oh * a.ow, g->stride * g->stride * g->c, kb * kb * g->cout,
                   precision);
}

// out[(q*C + c) * kb^2*Cout + (ty*kb + tx) * Cout + co]
//   = w[co][s (kb-1-ty) + q / s][s (kb-1-tx) + q % s][c]   (w in KRSC)
__global__ void dgrad_weights_kernel(const float* __restrict__ w, float* __restrict__ out,
                                     int cout, int k, int c, int s, int total) {
  pdl_trigger();
  pdl_wait();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int kb = k / s;
  const int co = idx % cout;
  int t = idx / cout;
  const int tx = t % kb;
  t /= kb;
  const int ty = t % kb;
  t /= kb;
  const int ch = t % c;
  const int q = t / c;
  const int ky = s * (kb - 1 - ty) + q / s;
  const int kx = s * (kb - 1 - tx) + q % s;
  out[idx] = w[((static_cast<long long>(co) * k + ky) * k + kx) * c + ch];
}

int conv_dgrad_weights(const float* w, float* out, const ttrl_conv_geom* g, cudaStream_t st) {
  int rc = check_conv(g);
  if (rc) return rc;
  if (!direct_dgrad_applies(g))
    return set_error(TTRL_EUNSUPPORTED, "conv_dgrad_weights: this geometry takes the column path");
  if (!w || !out) return set_error(TTRL_EINVAL, "conv_dgrad_weights: null pointer");
  const int total = g->kh * g->kw * g->c * g->cout;
  const cudaError_t le = launch_pdl(dgrad_weights_kernel, dim3((total + 255) / 256), dim3(256), 0,
                                    st, w, out, g->cout, g->kh, g->c, g->stride, total);
  note_launch();
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("dgrad weights launch", e);
}

size_t conv_dgrad_weights_bytes(const ttrl_conv_geom* g) {
  return direct_dgrad_applies(g) ? dgrad_weights_bytes(g) : 0;
}

size_t conv_dgrad_prepared_ws(const ttrl_conv_geom* g) {
  return direct_dgrad_applies(g) ? gemm_workspace_bytes(direct_dgrad_desc(g, TTRL_PREC_TF32X3))
                                 : 0;
}

// The sub-pixel GEMM over stacked sub-kernels `wt` (conv_dgrad_weights);
// workspace [counters | split-K partials].
int conv_dgrad_prepared(const float* dy, const float* wt, const float* mask, float* dx,
                        const ttrl_conv_geom* g, int accumulate, int precision, float* ws,
                        size_t wsb, int* status, cudaStream_t st) {
  int rc = check_conv(g);
  if (rc) return rc;
  if (!direct_dgrad_applies(g))
    return set_error(TTRL_EUNSUPPORTED, "conv_dgrad_prepared: this geometry takes the column path");
  const size_t need = conv_dgrad_prepared_ws(g);
  if (ws == nullptr || wsb < need)
    return set_error(TTRL_EWORKSPACE, "conv_dgrad_prepared: needs %zu bytes of workspace, got %zu",
                     need, wsb);
  const ttrl_conv_geom a = dgrad_window_geom(g);
  ttrl_gemm_desc d = direct_dgrad_desc(g, precision);
  d.a = conv_operand(dy, TTRL_OPND_CONV_FPROP, a);
  d.b = dense(wt, d.n, d.k, d.k, 1);
  d.ep = epi(dx, g->c, 1);
  d.ep.accumulate = accumulate;
  if (mask) {
    d.ep.mask = mask;
    d.ep.mrs = g->c;
    d.ep.mcs = 1;
  }
  EpiExtra ex = no_extra();
  if (g->stride > 1) {
    ex.scatter_s = g->stride;
    ex.scatter_c = g->c;
    ex.scatter_h = g->h;
    ex.scatter_w = g->w;
    ex.scatter_gh = a.oh;
    ex.scatter_gw = a.ow;
    ex.f_sc = make_fastdiv(g->c);
    ex.f_s = make_fastdiv(g->stride);
    ex.f_gw = make_fastdiv(a.ow);
    ex.f_ghw = make_fastdiv(a.oh * a.ow);
  }
  return gemm_run_ws(d, 0, ex, ws, wsb, status, st);
}

static int conv_dgrad_direct(const float* dy, const float* w, const float* mask, float* dx,
                             const ttrl_conv_geom* g, int accumulate, int precision, float* ws,
                             size_t wsb, int* status, cudaStream_t st) {
  const size_t wb = dgrad_weights_bytes(g);
  float* wt = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + kCounterBytes);
  int rc = conv_dgrad_weights(w, wt, g, st);
  if (rc) return rc;
  const ttrl_conv_geom a = dgrad_window_geom(g);
  ttrl_gemm_desc d = direct_dgrad_desc(g, precision);
  d.a = conv_operand(dy, TTRL_OPND_CONV_FPROP, a);
  d.b = dense(wt, d.n, d.k, d.k, 1);
  d.ep = epi(dx, g->c, 1);
  d.ep.accumulate = accumulate;
  if (mask) {
    d.ep.mask = mask;
    d.ep.mrs = g->c;
    d.ep.mcs = 1;
  }
  EpiExtra ex = no_extra();
  if (g->stride > 1) {
    ex.scatter_s = g->stride;
    ex.scatter_c = g->c;
    ex.scatter_h = g->h;
    ex.scatter_w = g->w;
    ex.scatter_gh = a.oh;
    ex.scatter_gw = a.ow;
    ex.f_sc = make_fastdiv(g->c);
    ex.f_s = make_fastdiv(g->stride);
    ex.f_gw = make_fastdiv(a.ow);
    ex.f_ghw = make_fastdiv(a.oh * a.ow);
  }
  char* partials = reinterpret_cast<char*>(wt) + wb;
  return gemm_run(d, 0, ex, reinterpret_cast<int*>(ws), reinterpret_cast<float*>(partials),
                  wsb - kCounterBytes - wb, status, st);
}

size_t conv_dgrad_ws(const ttrl_conv_geom* g) {
  if (direct_dgrad_applies(g)) {
    // [counters | stacked sub-kernels | the GEMM's split-K partials]
    return gemm_workspace_bytes(direct_dgrad_desc(g, TTRL_PREC_TF32X3)) + dgrad_weights_bytes(g);
  }
  const size_t m = static_cast<size_t>(g->n) * g->oh * g->ow;
  const size_t kk = static_cast<size_t>(g->kh) * g->kw * g->c;
  ttrl_gemm_desc d = make_desc(static_cast<int>(m), static_cast<int>(kk), g->cout,
                               TTRL_PREC_TF32X3);
  // [counters | column buffer | the GEMM's split-K partials]
  return gemm_workspace_bytes(d) + ((m * kk * sizeof(float) + 255) & ~static_cast<size_t>(255));
}

int conv_dgrad(const float* dy, const float* w, const float* mask, float* dx,
               const ttrl_conv_geom* g, int accumulate, int precision, float* ws, size_t wsb,
               int* status, cudaStream_t st) {
  int rc = check_conv(g);
  if (rc) return rc;
  const int m = g->n * g->oh * g->ow;
  const int kk = g->kh * g->kw * g->c;
  const size_t need = conv_dgrad_ws(g);
  if (ws == nullptr || wsb < need)
    return set_error(TTRL_EWORKSPACE, "conv_dgrad: needs %zu bytes of workspace, got %zu", need,
                     wsb);
  if (direct_dgrad_applies(g))
    return conv_dgrad_direct(dy, w, mask, dx, g, accumulate, precision, ws, wsb, status, st);
  const size_t col_bytes =
      (static_cast<size_t>(m) * kk * sizeof(float) + 255) & ~static_cast<size_t>(255);
  float* dxcol = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + kCounterBytes);
  ttrl_gemm_desc d = make_desc(m, kk, g->cout, precision);
  d.a = dense(dy, m, g->cout, g->cout, 1);
  d.b = dense(w, kk, g->cout, 1, kk);
  d.ep = epi(dxcol, kk, 1);
  rc = gemm_run(d, 0, no_extra(), reinterpret_cast<int*>(ws),
                reinterpret_cast<float*>(reinterpret_cast<char*>(dxcol) + col_bytes),
                wsb - kCounterBytes - col_bytes, status, st);
  if (rc) return rc;
  const int taps = ((g->kh + g->stride - 1) / g->stride) * ((g->kw + g->stride - 1) / g->stride);
  if (taps > kCol2imMaxTaps)
    return set_error(TTRL_EUNSUPPORTED, "conv_dgrad: %d kernel taps per input pixel exceed %d",
                     taps, kCol2imMaxTaps);
  Col2imArgs a;
  std::memset(&a, 0, sizeof(a));
  a.dxcol = dxcol;
  a.mask = mask;
  a.dx = dx;
  a.g = *g;
  const bool vec = g->c % 4 == 0 && (reinterpret_cast<uintptr_t>(dx) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(mask) & 15u) == 0;
  a.vec = vec ? 1 : 0;
  a.cg = vec ? g->c / 4 : g->c;
  a.f_cg = make_fastdiv(a.cg);
  a.f_w = make_fastdiv(g->w);
  a.f_h = make_fastdiv(g->h);
  a.f_s = make_fastdiv(g->stride);
  a.accumulate = accumulate;
  const long long total = static_cast<long long>(g->n) * g->h * g->w * a.cg;
  if (total >= (1ll << 31)) return set_error(TTRL_EUNSUPPORTED, "conv_dgrad: input too large");
  a.total = static_cast<int>(total);
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  cudaError_t le_;
  if (vec)
    le_ = launch_pdl(col2im_kernel<true>, dim3(blocks), dim3(256), 0, st, a);
  else
    le_ = launch_pdl(col2im_kernel<false>, dim3(blocks), dim3(256), 0, st, a);
  note_launch();
  cudaError_t e = le_ != cudaSuccess ? le_ : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("col2im launch", e);
}

// The stream-K weight gradient is on unless TTRL_WGRAD_SK=0 (which keeps
// the general GEMM, for comparisons).
static bool wgrad_sk_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("TTRL_WGRAD_SK");
    return e == nullptr || std::atoi(e) != 0;
  }();
  return on;
}

size_t conv_wgrad_ws(const ttrl_conv_geom* g) {
  const int m = g->n * g->oh * g->ow;
  const int kk = g->kh * g->kw * g->c;
  ttrl_gemm_desc d = make_desc(kk + 1, g->cout, m, TTRL_PREC_TF32X3);
  const size_t generic = gemm_workspace_bytes(d);
  if (wgrad_sk_geometry(g) && wgrad_sk_enabled()) {
    const size_t sk = wgrad_sk_ws(g);
    return sk > generic ? sk : generic;
  }
  return generic;
}

int conv_wgrad(const float* x, const float* dy, float* dw, float* db, const ttrl_conv_geom* g,
               float alpha, int accumulate, int accumulate_db, int precision, float* ws,
               size_t wsb, int* status, cudaStream_t st) {
  int rc = check_conv(g);
  if (rc) return rc;
  if (wgrad_sk_enabled() && wgrad_sk_applies(g, x, dy)) {
    // EUNSUPPORTED (no TMA map for these operands) is refused before any
    // launch; the general GEMM then takes the call.
    rc = wgrad_sk_run(x, dy, dw, db, g, alpha, accumulate, accumulate_db, precision, ws, wsb,
                      status, st);
    if (rc != TTRL_EUNSUPPORTED) return rc;
  }
  const int m = g->n * g->oh * g->ow;
  const int kk = g->kh * g->kw * g->c;
  ttrl_gemm_desc d = make_desc(kk + (db ? 1 : 0), g->cout, m, precision);
  d.a = conv_operand(x, TTRL_OPND_CONV_WGRAD, *g);
  d.b = dense(dy, g->cout, m, 1, g->cout);
  d.ep = epi(dw, 1, kk);
  d.ep.alpha = alpha;
  d.ep.accumulate = accumulate;
  EpiExtra ex = no_extra();
  if (db) {
    // db (not scaled by alpha) as an extra row of ones appended to the
    // windows operand: its row of D is the column sums of dY.
    ex.row2 = kk;
    ex.out2 = db;
    ex.cs2 = 1;
    ex.accumulate2 = accumulate_db;
  }
  return gemm_run_ws(d, db ? 1 : 0, ex, ws, wsb, status, st);
}

// ------------------------------------------------------- frame conversion

__global__ void u8_nchw_to_f32_nhwc_kernel(const uint8_t* __restrict__ in,
                                           const int32_t* __restrict__ index,
                                           float* __restrict__ out, int n, int c, int h, int w,
                                           float scale, FastDiv f_hw) {
  pdl_trigger();
  pdl_wait();
  const int pixels = n * h * w;
  const int hw = h * w;
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < pixels; p += gridDim.x * blockDim.x) {
    const int img = fdiv(f_hw, p);
    const int pix = p - img * hw;
    const int src = index ? index[img] : img;
    const uint8_t* base = in + static_cast<long long>(src) * c * hw + pix;
    float* o = out + p * c;
    if (c == 4) {
      float4 v = make_float4(base[0] * scale, base[hw] * scale, base[2 * hw] * scale,
                             base[3 * hw] * scale);
      *reinterpret_cast<float4*>(o) = v;
    } else {
      for (int ch = 0; ch < c; ++ch) o[ch] = base[static_cast<long long>(ch) * hw] * scale;
    }
  }
}

int u8_to_f32(const uint8_t* in, const int32_t* index, float* out, int n, int c, int h, int w,
              float scale, cudaStream_t st) {
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0) return set_error(TTRL_EINVAL, "u8_to_f32: bad extents");
  if (in == nullptr || out == nullptr) return set_error(TTRL_EINVAL, "u8_to_f32: null pointer");
  if (c == 4 && (reinterpret_cast<uintptr_t>(out) & 15u))
    return set_error(TTRL_EINVAL, "u8_to_f32: output must be 16-byte aligned");
  const long long pixels = static_cast<long long>(n) * h * w;
  int blocks = static_cast<int>((pixels + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (pixels * static_cast<long long>(c) >= (1ll << 31))
    return set_error(TTRL_EUNSUPPORTED, "u8_to_f32: more than 2^31 values");
  const cudaError_t le_ = launch_pdl(u8_nchw_to_f32_nhwc_kernel, dim3(blocks), dim3(256), 0, st, in, index, out, n, c, h, w, scale,
                                                      make_fastdiv(h * w));
  note_launch();
  cudaError_t e = le_ != cudaSuccess ? le_ : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("u8_to_f32 launch", e);
}

// Frames to space-to-depth rows: out[(img, Y, X)][(dy * f + dx) * c + ch] =
// in[src][ch][Y * f + dy][X * f + dx] * scale, the input layout of a
// stride-f convolution whose kernel f divides, rewritten as a stride-1
// convolution over f*f*c channels (the same products, in another order).
// One thread per (img, Y, dy, X) when c == 4 and f == 4: four 4-byte loads
// (one per channel) and four float4 stores.
__global__ void u8_nchw_to_f32_s2d_kernel(const uint8_t* __restrict__ in,
                                          const int32_t* __restrict__ index,
                                          float* __restrict__ out, int n, int c, int h, int w,
                                          int f, float scale) {
  pdl_trigger();
  pdl_wait();
  const int hf = h / f, wf = w / f, hw = h * w;
  const int cc = f * f * c;
  if (c == 4 && f == 4) {
    const long long items = static_cast<long long>(n) * hf * f * wf;
    for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < items;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
      const int X = static_cast<int>(t % wf);
      long long r = t / wf;
      const int dy = static_cast<int>(r % f);
      r /= f;
      const int Y = static_cast<int>(r % hf);
      const int img = static_cast<int>(r / hf);
      const int src = index ? index[img] : img;
      const uint8_t* base = in + static_cast<long long>(src) * c * hw +
                            static_cast<long long>(Y * f + dy) * w + X * f;
      uchar4 px[4];
#pragma unroll
      for (int ch = 0; ch < 4; ++ch)
        px[ch] = *reinterpret_cast<const uchar4*>(base + static_cast<long long>(ch) * hw);
      float* o = out + ((static_cast<long long>(img) * hf + Y) * wf + X) * cc + dy * f * c;
      const float4 v0 = make_float4(px[0].x * scale, px[1].x * scale, px[2].x * scale, px[3].x * scale);
      const float4 v1 = make_float4(px[0].y * scale, px[1].y * scale, px[2].y * scale, px[3].y * scale);
      const float4 v2 = make_float4(px[0].z * scale, px[1].z * scale, px[2].z * scale, px[3].z * scale);
      const float4 v3 = make_float4(px[0].w * scale, px[1].w * scale, px[2].w * scale, px[3].w * scale);
      reinterpret_cast<float4*>(o)[0] = v0;
      reinterpret_cast<float4*>(o)[1] = v1;
      reinterpret_cast<float4*>(o)[2] = v2;
      reinterpret_cast<float4*>(o)[3] = v3;
    }
    return;
  }
  const long long total = static_cast<long long>(n) * hf * wf * cc;
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(t % cc);
    const long long pix = t / cc;
    const int X = static_cast<int>(pix % wf);
    const long long r = pix / wf;
    const int Y = static_cast<int>(r % hf);
    const int img = static_cast<int>(r / hf);
    const int ch = k % c, dd = k / c, dx = dd % f, dy = dd / f;
    const int src = index ? index[img] : img;
    out[t] = in[static_cast<long long>(src) * c * hw + static_cast<long long>(ch) * hw +
                static_cast<long long>(Y * f + dy) * w + X * f + dx] * scale;
  }
}

int u8_to_f32_s2d(const uint8_t* in, const int32_t* index, float* out, int n, int c, int h, int w,
                  int f, float scale, cudaStream_t st) {
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0 || f <= 0)
    return set_error(TTRL_EINVAL, "u8_to_f32_s2d: bad extents");
  if (h % f || w % f) return set_error(TTRL_EINVAL, "u8_to_f32_s2d: fold %d must divide %dx%d", f, h, w);
  if (in == nullptr || out == nullptr) return set_error(TTRL_EINVAL, "u8_to_f32_s2d: null pointer");
  const bool fast = c == 4 && f == 4;
  if (fast && ((reinterpret_cast<uintptr_t>(out) & 15u) || (reinterpret_cast<uintptr_t>(in) & 3u) ||
               (w & 3) || ((h * w) & 3)))
    return set_error(TTRL_EINVAL, "u8_to_f32_s2d: unaligned frames or output");
  const long long values = static_cast<long long>(n) * h * w * c;
  if (values >= (1ll << 31)) return set_error(TTRL_EUNSUPPORTED, "u8_to_f32_s2d: more than 2^31 values");
  const long long items = fast ? values / 16 : values;
  int blocks = static_cast<int>((items + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  const cudaError_t le_ = launch_pdl(u8_nchw_to_f32_s2d_kernel, dim3(blocks), dim3(256), 0, st, in,
                                     index, out, n, c, h, w, f, scale);
  note_launch();
  cudaError_t e = le_ != cudaSuccess ? le_ : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("u8_to_f32_s2d launch", e);
}

}  // namespace ttrl
