// tcgen05 GEMM for the learner update: D[r][c] = sum_k A[r][k] * B[c][k].
//
// One CTA (4 warps) owns a 128 x BN tile of D held in TMEM and walks its
// share of K in 32-wide k-blocks through a cp.async ring of shared-memory
// stages. Each operand is *gathered* (dense strided matrix, convolution
// im2col, or transposed im2col for the weight gradient), so one kernel
// serves Linear fwd/dgrad/wgrad and Conv2d fprop/dgrad/wgrad without
// materialising any im2col buffer. Tiles land in the canonical 128-byte
// swizzled layout, K-major or MN-major depending on which dimension is
// contiguous in global memory, and thread 0 issues tcgen05.mma.kind::tf32.
//
// Precision: TTRL_PREC_TF32X3 splits every operand into a tf32 high part and
// an fp32 remainder in shared memory and accumulates hi*hi + hi*lo + lo*hi,
// which reproduces fp32 products to ~1e-6 relative. TTRL_PREC_TF32 issues a
// single pass on the truncated operands.
//
// K can be split across CTAs (blockIdx.z); partial tiles then go to a
// caller workspace and a second kernel sums them in split order, so the
// result is deterministic from run to run.
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace ttrl {

// Constant sources for the synthetic "ones" row an operand may append: a
// GEMM whose A operand carries a row of ones produces the column sums of B
// (the bias gradient) in that row of D.
__device__ __align__(16) float kOnes4[4] = {1.f, 1.f, 1.f, 1.f};
__device__ __align__(16) float kOneZeros[4] = {1.f, 0.f, 0.f, 0.f};

__device__ __forceinline__ const float* opnd_addr(const DevOperand& o, int r, int k, bool& ok) {
  ok = false;
  if (k >= o.kdim) return o.ptr;
  if (r >= o.rows) {
    if (o.ones_row && r == o.rows) {
      ok = true;
      return o.mode == 1 ? kOneZeros : kOnes4;
    }
    return o.ptr;
  }
  if (o.kind == TTRL_OPND_DENSE) {
    ok = true;
    return o.ptr + static_cast<long long>(r) * o.rs + static_cast<long long>(k) * o.ks;
  }
  int m, q;
  if (o.kind == TTRL_OPND_CONV_FPROP) {
    m = r;
    q = k;
  } else {
    m = k;
    q = r;
  }
  const int ohw = o.oh * o.ow;
  const int img = m / ohw;
  const int rem = m - img * ohw;
  const int oy = rem / o.ow;
  const int ox = rem - oy * o.ow;
  const int c = q % o.c;
  const int t = q / o.c;
  const int kx = t % o.kw;
  const int ky = t / o.kw;
  const int iy = oy * o.stride - o.pad + ky;
  const int ix = ox * o.stride - o.pad + kx;
  if (iy < 0 || iy >= o.h || ix < 0 || ix >= o.w) return o.ptr;
  ok = true;
  return o.ptr + ((static_cast<long long>(img) * o.h + iy) * o.w + ix) * o.c + c;
}

// Gather one [R rows x 32 k] tile of operand `o` into shared memory at
// `base` (1024-byte aligned). Issues cp.async copies only; the caller
// commits and waits.
template <int R>
__device__ __forceinline__ void load_tile(const DevOperand& o, uint32_t base, int row0, int k0,
                                          int tid) {
  constexpr int NT = 128;
  if (o.mode == kModeKVec) {
#pragma unroll 4
    for (int t = tid; t < R * 8; t += NT) {
      const int r = t >> 3, kc = t & 7;
      bool ok;
      const float* src = opnd_addr(o, row0 + r, k0 + kc * 4, ok);
      cp_async16(base + kmajor_off(r, kc * 4), src, ok ? 16u : 0u);
    }
  } else if (o.mode == kModeMNVec) {
    constexpr int RC = R / 4;
#pragma unroll 4
    for (int t = tid; t < RC * 32; t += NT) {
      const int rc = t % RC, k = t / RC;
      bool ok;
      const float* src = opnd_addr(o, row0 + rc * 4, k0 + k, ok);
      cp_async16(base + mnmajor_off(rc * 4, k), src, ok ? 16u : 0u);
    }
  } else if (o.mode == kModeScalarK) {
#pragma unroll 4
    for (int t = tid; t < R * 32; t += NT) {
      const int r = t >> 5, k = t & 31;
      bool ok;
      const float* src = opnd_addr(o, row0 + r, k0 + k, ok);
      cp_async4(base + kmajor_off(r, k), src, ok ? 4u : 0u);
    }
  } else {  // kModeScalarR: rows fastest across threads
#pragma unroll 4
    for (int t = tid; t < R * 32; t += NT) {
      const int r = t % R, k = t / R;
      bool ok;
      const float* src = opnd_addr(o, row0 + r, k0 + k, ok);
      cp_async4(base + kmajor_off(r, k), src, ok ? 4u : 0u);
    }
  }
}

__device__ __forceinline__ void epi_store(const ttrl_epilogue& ep, const EpiExtra& ex, int r,
                                          int c, float acc) {
  if (ex.row2 >= 0 && r == ex.row2) {
    // The synthetic ones row: column sums of B, stored unscaled.
    float* o = ex.out2 + static_cast<long long>(c) * ex.cs2;
    float v = acc;
    if (ex.accumulate2) v += *o;
    *o = v;
    return;
  }
  float v = ep.alpha * acc;
  if (ep.bias_mode == TTRL_BIAS_ROW) {
    v += ep.bias[r];
  } else if (ep.bias_mode == TTRL_BIAS_COL) {
    v += ep.bias[c];
  }
  if (ep.mask != nullptr) {
    if (!(ep.mask[static_cast<long long>(r) * ep.mrs + static_cast<long long>(c) * ep.mcs] > 0.f))
      v = 0.f;
  }
  if (ep.relu) v = v > 0.f ? v : 0.f;
  float* o = ep.out + static_cast<long long>(r) * ep.ors + static_cast<long long>(c) * ep.ocs;
  if (ep.accumulate) v += *o;
  *o = v;
}

template <int BN, bool SPLIT>
struct TileCfg {
  static constexpr int kABytes = 128 * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kTile = kABytes + kBBytes;
  static constexpr int kStage = kTile * (SPLIT ? 2 : 1);
  static constexpr int kStagesRaw = (196 * 1024) / kStage;
  static constexpr int kStages = kStagesRaw > 4 ? 4 : kStagesRaw;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kSmem = kStages * kStage + 1024 /*align slack*/ + 256 /*barriers*/;
  static_assert(kStages >= 2, "at least two pipeline stages");
};

template <int BN, bool SPLIT>
__global__ void __launch_bounds__(128, 1) gemm_tc_kernel(const __grid_constant__ GemmArgs args) {
  using Cfg = TileCfg<BN, SPLIT>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t sbase = (raw_u32 + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - raw_u32);
  const uint32_t bar0 = sbase + S * Cfg::kStage;  // S "stage free" barriers
  const uint32_t accum_bar = bar0 + S * 8;
  const uint32_t tmem_slot = accum_bar + 8;
  const uint32_t* tmem_slot_gen =
      reinterpret_cast<const uint32_t*>(sgen + (tmem_slot - sbase));

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (warp == 0) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(bar0 + s * 8, 1);
    mbar_init(accum_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot_gen;

  const int row0 = blockIdx.x * 128;
  const int col0 = blockIdx.y * BN;
  const int kb0 = blockIdx.z * args.kb_per_split;
  const int kb1 = min(args.kblocks, kb0 + args.kb_per_split);
  const int nk = kb1 - kb0;
  const bool a_mn = args.a.mode == kModeMNVec;
  const bool b_mn = args.b.mode == kModeMNVec;
  const uint32_t idesc = idesc_tf32(128, BN, a_mn, b_mn);
  bool timed_out = false;

  auto stage_a = [&](int s) { return sbase + s * Cfg::kStage; };
  auto stage_b = [&](int s) { return sbase + s * Cfg::kStage + Cfg::kABytes; };

  // Prologue: put S-1 k-blocks in flight.
#pragma unroll 1
  for (int s = 0; s < S - 1; ++s) {
    if (s < nk) {
      load_tile<128>(args.a, stage_a(s), row0, (kb0 + s) * 32, tid);
      load_tile<BN>(args.b, stage_b(s), col0, (kb0 + s) * 32, tid);
    }
    cp_async_commit();
  }

#pragma unroll 1
  for (int i = 0; i < nk; ++i) {
    const int j = i + S - 1;
    if (j < nk) {
      const int sj = j % S;
      if (i >= 1) {
        // Stage sj was last read by the MMAs of k-block i-1.
        if (!mbar_wait(bar0 + sj * 8, ((i - 1) / S) & 1)) timed_out = true;
      }
      load_tile<128>(args.a, stage_a(sj), row0, (kb0 + j) * 32, tid);
      load_tile<BN>(args.b, stage_b(sj), col0, (kb0 + j) * 32, tid);
    }
    cp_async_commit();
    cp_async_wait<S - 1>();
    __syncthreads();
    const int s = i % S;
    if constexpr (SPLIT) {
      // hi = x with the low 13 mantissa bits cleared, written back in place
      // so the tensor core sees an exact tf32 value; lo = x - hi.
      uint8_t* st = sgen + s * Cfg::kStage;
#pragma unroll 4
      for (int off = tid * 16; off < Cfg::kTile; off += 128 * 16) {
        float4 x = *reinterpret_cast<float4*>(st + off);
        float4 hi, lo;
        split_tf32(x.x, hi.x, lo.x);
        split_tf32(x.y, hi.y, lo.y);
        split_tf32(x.z, hi.z, lo.z);
        split_tf32(x.w, hi.w, lo.w);
        *reinterpret_cast<float4*>(st + off) = hi;
        *reinterpret_cast<float4*>(st + Cfg::kTile + off) = lo;
      }
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t a_hi = stage_a(s), b_hi = stage_b(s);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        // One MMA consumes k = 8: 32 bytes along a K-major line, or two
        // 512-byte k-groups of an MN-major tile.
        const uint32_t aoff = a_mn ? ks * 1024u : ks * 32u;
        const uint32_t boff = b_mn ? ks * 1024u : ks * 32u;
        const uint32_t albo = a_mn ? 4096u : 16u, blbo = b_mn ? 4096u : 16u;
        const uint32_t asbo = a_mn ? 512u : 1024u, bsbo = b_mn ? 512u : 1024u;
        const uint32_t alay = a_mn ? kLayoutSw128Base32 : kLayoutSw128;
        const uint32_t blay = b_mn ? kLayoutSw128Base32 : kLayoutSw128;
        const uint64_t ad = umma_desc(a_hi + aoff, albo, asbo, alay);
        const uint64_t bd = umma_desc(b_hi + boff, blbo, bsbo, blay);
        umma_tf32(tmem, ad, bd, idesc, (i > 0 || ks > 0) ? 1u : 0u);
        if constexpr (SPLIT) {
          const uint64_t adl = umma_desc(a_hi + Cfg::kTile + aoff, albo, asbo, alay);
          const uint64_t bdl = umma_desc(b_hi + Cfg::kTile + boff, blbo, bsbo, blay);
          umma_tf32(tmem, ad, bdl, idesc, 1u);
          umma_tf32(tmem, adl, bd, idesc, 1u);
        }
      }
      umma_commit(bar0 + s * 8);
    }
  }

  if (tid == 0) umma_commit(accum_bar);
  if (!mbar_wait(accum_bar, 0)) timed_out = true;
  tc_fence_after();

  if (timed_out) {
    record_error(args.status, kErrWaitTimeout);
  } else {
    // Epilogue: warp w reads TMEM lanes [32w, 32w+32) = tile rows.
    const int r = row0 + warp * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < BN; c += 8) {
      if (col0 + c >= args.n) break;  // uniform across the warp
      float v[8];
      tmem_ld8(trow + c, v);
      if (r < args.m) {
        if (args.ws != nullptr) {
          float* w = args.ws + (static_cast<long long>(blockIdx.z) * args.m + r) * args.n;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (col0 + c + q < args.n) w[col0 + c + q] = v[q];
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            if (col0 + c + q < args.n) epi_store(args.ep, args.ex, r, col0 + c + q, v[q]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, Cfg::kTmemCols);
}

// Sum split-K partials in split order and apply the epilogue.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int m, int n,
                                     ttrl_epilogue ep, EpiExtra ex) {
  const long long total = static_cast<long long>(m) * n;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(idx / n);
    const int c = static_cast<int>(idx - static_cast<long long>(r) * n);
    float s = 0.f;
    for (int sp = 0; sp < splits; ++sp) s += ws[static_cast<long long>(sp) * total + idx];
    epi_store(ep, ex, r, c, s);
  }
}

// ------------------------------------------------------------------ host

template <int BN, bool SPLIT>
static int set_smem_attr() {
  using Cfg = TileCfg<BN, SPLIT>;
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, SPLIT>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("cudaFuncSetAttribute(gemm)", e);
}

int gemm_init_device() {
  int rc = TTRL_OK;
  if ((rc = set_smem_attr<32, true>())) return rc;
  if ((rc = set_smem_attr<64, true>())) return rc;
  if ((rc = set_smem_attr<128, true>())) return rc;
  if ((rc = set_smem_attr<256, true>())) return rc;
  if ((rc = set_smem_attr<32, false>())) return rc;
  if ((rc = set_smem_attr<64, false>())) return rc;
  if ((rc = set_smem_attr<128, false>())) return rc;
  if ((rc = set_smem_attr<256, false>())) return rc;
  return TTRL_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Pick the gather mode of an operand from its strides and alignment.
static int resolve_operand(const ttrl_operand& in, int ones_row, DevOperand& out) {
  std::memset(&out, 0, sizeof(out));
  out.ptr = static_cast<const float*>(in.ptr);
  out.kind = in.kind;
  out.rows = in.rows;
  out.kdim = in.kdim;
  out.rs = in.rs;
  out.ks = in.ks;
  out.n = in.n;
  out.h = in.h;
  out.w = in.w;
  out.c = in.c;
  out.kh = in.kh;
  out.kw = in.kw;
  out.stride = in.stride;
  out.pad = in.pad;
  out.oh = in.oh;
  out.ow = in.ow;
  out.ones_row = ones_row;
  if (in.ptr == nullptr && in.rows > 0 && in.kdim > 0)
    return set_error(TTRL_EINVAL, "gemm operand has a null pointer");
  if (in.kind == TTRL_OPND_DENSE) {
    const bool al = aligned16(in.ptr);
    if (in.ks == 1 && in.kdim % 4 == 0 && in.rs % 4 == 0 && al) {
      out.mode = kModeKVec;
    } else if (in.rs == 1 && in.rows % 4 == 0 && in.ks % 4 == 0 && al) {
      out.mode = kModeMNVec;
    } else {
      out.mode = (in.rs <= in.ks && in.rs != 0) ? kModeScalarR : kModeScalarK;
    }
    return TTRL_OK;
  }
  if (in.kind == TTRL_OPND_CONV_FPROP || in.kind == TTRL_OPND_CONV_WGRAD) {
    if (in.n <= 0 || in.h <= 0 || in.w <= 0 || in.c <= 0 || in.kh <= 0 || in.kw <= 0 ||
        in.stride <= 0 || in.pad < 0 || in.oh <= 0 || in.ow <= 0)
      return set_error(TTRL_EINVAL, "gemm conv operand has an invalid geometry");
    const bool vec = (in.c % 4 == 0) && aligned16(in.ptr);
    if (in.kind == TTRL_OPND_CONV_FPROP)
      out.mode = vec ? kModeKVec : kModeScalarK;
    else
      out.mode = vec ? kModeMNVec : kModeScalarR;
    return TTRL_OK;
  }
  return set_error(TTRL_EINVAL, "gemm operand kind %d is unknown", in.kind);
}

static int pick_bn(int n) {
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  if (n <= 128) return 128;
  return 256;
}

struct Schedule {
  int bn, kblocks, splits, kb_per_split, tiles;
};

static Schedule make_schedule(const ttrl_gemm_desc& d) {
  Schedule s;
  s.bn = pick_bn(d.n);
  s.kblocks = (d.k + 31) / 32;
  s.tiles = ((d.m + 127) / 128) * ((d.n + s.bn - 1) / s.bn);
  int splits = d.splits;
  if (splits <= 0) {
    // Aim for about one wave of 148 SMs with at least 4 k-blocks per CTA.
    splits = 1;
    if (s.tiles < 100 && s.kblocks >= 8) {
      const int want = (148 + s.tiles - 1) / s.tiles;
      const int most = s.kblocks / 4;
      splits = want < most ? want : most;
      if (splits < 1) splits = 1;
    }
  }
  if (splits > s.kblocks) splits = s.kblocks > 0 ? s.kblocks : 1;
  s.kb_per_split = (s.kblocks + splits - 1) / splits;
  if (s.kb_per_split < 1) s.kb_per_split = 1;
  s.splits = (s.kblocks + s.kb_per_split - 1) / s.kb_per_split;
  if (s.splits < 1) s.splits = 1;
  return s;
}

size_t gemm_workspace_bytes(const ttrl_gemm_desc& d) {
  const Schedule s = make_schedule(d);
  if (s.splits <= 1) return 0;
  return static_cast<size_t>(s.splits) * d.m * d.n * sizeof(float);
}

template <int BN, bool SPLIT>
static cudaError_t launch_bn(const GemmArgs& args, dim3 grid, cudaStream_t stream) {
  using Cfg = TileCfg<BN, SPLIT>;
  gemm_tc_kernel<BN, SPLIT><<<grid, 128, Cfg::kSmem, stream>>>(args);
  return cudaGetLastError();
}

int gemm_run(const ttrl_gemm_desc& d, int a_ones_row, const EpiExtra& ex, float* ws,
             size_t ws_bytes, int* status, cudaStream_t stream) {
  if (d.m < 0 || d.n < 0 || d.k < 0) return set_error(TTRL_EINVAL, "gemm: negative extent");
  if (d.m == 0 || d.n == 0) return TTRL_OK;
  if (d.ep.out == nullptr) return set_error(TTRL_EINVAL, "gemm: null output");
  if (d.precision != TTRL_PREC_TF32X3 && d.precision != TTRL_PREC_TF32)
    return set_error(TTRL_EINVAL, "gemm: unknown precision %d", d.precision);
  if (d.k == 0) return set_error(TTRL_EUNSUPPORTED, "gemm: empty reduction (k == 0)");

  GemmArgs args;
  std::memset(&args, 0, sizeof(args));
  int rc;
  if ((rc = resolve_operand(d.a, a_ones_row, args.a))) return rc;
  if ((rc = resolve_operand(d.b, 0, args.b))) return rc;
  if (args.a.rows + (a_ones_row ? 1 : 0) < d.m || args.b.rows < d.n)
    return set_error(TTRL_EINVAL, "gemm: operand rows smaller than the output extent");
  args.ep = d.ep;
  args.ex = ex;
  args.m = d.m;
  args.n = d.n;
  args.k = d.k;
  args.status = status;

  const Schedule s = make_schedule(d);
  args.kblocks = s.kblocks;
  args.kb_per_split = s.kb_per_split;
  if (s.splits > 1) {
    const size_t need = static_cast<size_t>(s.splits) * d.m * d.n * sizeof(float);
    if (ws == nullptr || ws_bytes < need)
      return set_error(TTRL_EWORKSPACE, "gemm: needs %zu bytes of workspace, got %zu", need,
                       ws_bytes);
    args.ws = ws;
  }
  dim3 grid((d.m + 127) / 128, (d.n + s.bn - 1) / s.bn, s.splits);
  const bool split3 = d.precision == TTRL_PREC_TF32X3;
  cudaError_t e;
  switch (s.bn) {
    case 32: e = split3 ? launch_bn<32, true>(args, grid, stream) : launch_bn<32, false>(args, grid, stream); break;
    case 64: e = split3 ? launch_bn<64, true>(args, grid, stream) : launch_bn<64, false>(args, grid, stream); break;
    case 128: e = split3 ? launch_bn<128, true>(args, grid, stream) : launch_bn<128, false>(args, grid, stream); break;
    default: e = split3 ? launch_bn<256, true>(args, grid, stream) : launch_bn<256, false>(args, grid, stream); break;
  }
  if (e != cudaSuccess) return set_cuda_error("gemm launch", e);
  if (s.splits > 1) {
    const long long total = static_cast<long long>(d.m) * d.n;
    int blocks = static_cast<int>((total + 255) / 256);
    if (blocks > 148 * 8) blocks = 148 * 8;
    splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(ws, s.splits, d.m, d.n, d.ep, ex);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("gemm split-k reduce launch", e);
  }
  return TTRL_OK;
}

}  // namespace ttrl
