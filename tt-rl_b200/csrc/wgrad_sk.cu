// Stream-K weight gradient of a convolution whose input needs no tf32 split
// (the first layer, reading raw 0..255 pixels):
//
//   D[r][c] = sum over output pixels k of A[r][k] * dY[k][c]
//   A[r][k] = x at pixel k's window, filter tap and channel r = (tap, channel)
//   dW[c][r] = alpha * D[r][c],  db[c] = sum over k of dY[k][c]
//
// The reduction runs over every output pixel of the batch (102,400 at the
// Nature CNN's first layer, batch 256), while D is small (256 x 32). The
// general GEMM kernel tiles D into 128-row tiles and splits K per tile; here
// one CTA per SM owns a contiguous slice of K for ALL of D at once:
//   - MT 128-row accumulators live in TMEM side by side, so each k-block's
//     dY tile is loaded once and feeds all of them;
//   - the windows operand arrives by TMA im2col mode (one 32-channel x
//     32-pixel box per 32 rows), dY by a tiled TMA map, both into a ring of
//     stages that one producer thread refills as the MMAs drain them;
//   - four loader warps write dY's tf32 low part (split-TF32) or round dY to
//     tf32 (single pass) in shared memory, and while they have each element
//     in a register they add it into per-column sums: the bias gradient,
//     with no ones row and no extra tile;
//   - one MMA thread issues tcgen05.mma.kind::tf32 for every accumulator.
// Each CTA stores its partial D and partial column sums; a second kernel
// sums the partials in CTA order (a fixed order, so results repeat bit for
// bit) and applies alpha and the accumulate flags.
//
// Every wait is bounded (common.cuh); a wait that runs out records
// kErrWaitTimeout in the status word and the kernel finishes without
// hanging.
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace ttrl {

namespace {

constexpr int kSkLoaderWarps = 4;
constexpr int kSkLoaders = kSkLoaderWarps * 32;
constexpr int kSkProducerWarp = kSkLoaderWarps;
constexpr int kSkMmaWarp = kSkLoaderWarps + 1;
constexpr int kSkThreads = (kSkLoaderWarps + 2) * 32;

// One k-block of the windows operand, MN-major: R rows of (tap, channel) in
// groups of 32 (one TMA im2col box of 32 channels x 32 pixels each, 4 KB
// apart), pixels k0 .. k0+31. Groups past the last row repeat the last tap
// (those rows of D are never read).
template <int R>
__device__ __forceinline__ void tma_windows_mn(const CUtensorMap* map, const DevOperand& o,
                                               uint32_t dst, int k0, uint32_t bar) {
  const int img = fdiv(o.f_ohw, k0);
  const int pix = k0 - img * o.oh * o.ow;
  const int oy = fdiv(o.f_ow, pix);
  const int ox = pix - oy * o.ow;
  const int last = o.kh * o.kw - 1;
#pragma unroll
  for (int g = 0; g < R / 32; ++g) {
    int t = fdiv(o.f_c, g * 32);
    const int c = g * 32 - t * o.c;
    if (t > last) t = last;
    const int ky = fdiv(o.f_kw, t);
    tma_load_im2col_4d(dst + g * 4096, map, c, ox * o.stride - o.pad, oy * o.stride - o.pad, img,
                       static_cast<uint16_t>(t - ky * o.kw), static_cast<uint16_t>(ky), bar);
  }
}

template <int MT, int BN>
struct SkCfg {
  static constexpr int kABytes = MT * 128 * 128;  // MT x 128 rows x 32 k fp32
  static constexpr int kBBytes = BN * 128;        // BN rows x 32 k fp32
  static constexpr int kStageBytes = kABytes + 2 * kBBytes;  // + dY's low part
  static constexpr int kFit = (225 * 1024) / kStageBytes;
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  static constexpr int kTmemCols = MT * BN <= 32 ? 32 : MT * BN <= 64 ? 64
                                   : MT * BN <= 128 ? 128 : 256;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
  static_assert(kStages >= 3, "at least three pipeline stages");
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
};

struct WgradSkArgs {
  CUtensorMap tma_a;  // im2col map of x: 32 channels x 32 pixels per box
  CUtensorMap tma_b;  // tiled map of dY: 32 output channels x 32 pixels per box
  DevOperand a;       // x's convolution geometry (window origins per pixel)
  int32_t kblocks;    // 32-pixel blocks of the reduction
  int32_t ctas;       // CTAs (K slices)
  int32_t split;      // 1: split-TF32 (dY's low part), 0: one pass over rounded dY
  int32_t pad0;
  float* partial;     // [ctas][MT * 128][BN]
  float* partial_db;  // [ctas][BN]
  int* status;
};

template <int MT, int BN>
__global__ void __launch_bounds__(kSkThreads, 1)
    wgrad_sk_kernel(const __grid_constant__ WgradSkArgs args) {
  using Cfg = SkCfg<MT, BN>;
  constexpr int S = Cfg::kStages;
  constexpr int SLICES = kSkLoaders / BN;
  extern __shared__ uint8_t smem_raw[];
  __shared__ float s_cols[SLICES][BN];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t sbase = (raw_u32 + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - raw_u32);
  const uint32_t bar0 = sbase + S * Cfg::kStageBytes;
  const uint32_t tfull0 = bar0;           // S: the stage's TMA bytes landed
  const uint32_t ready0 = bar0 + S * 8;   // S: dY's low part written (loader warps)
  const uint32_t empty0 = bar0 + 2 * S * 8;  // S: the MMAs reading the stage are done
  const uint32_t accum_bar = bar0 + 3 * S * 8;
  const uint32_t tmem_slot = accum_bar + 8;
  const uint32_t* tmem_slot_gen = reinterpret_cast<const uint32_t*>(sgen + (tmem_slot - sbase));

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (warp == kSkMmaWarp) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  if (warp == kSkProducerWarp && lane == 0) {
    prefetch_tensormap(&args.tma_a);
    prefetch_tensormap(&args.tma_b);
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(tfull0 + s * 8, 1);
      mbar_init(ready0 + s * 8, kSkLoaderWarps);
      mbar_init(empty0 + s * 8, 1);
    }
    mbar_init(accum_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // This CTA's k-blocks: the first (kblocks % ctas) CTAs take one extra.
  const int z = blockIdx.x;
  const int q = args.kblocks / args.ctas, rem = args.kblocks % args.ctas;
  const int kb0 = z * q + min(z, rem);
  const int nk = q + (z < rem ? 1 : 0);
  bool timed_out = false;

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot_gen;
  pdl_trigger();
  pdl_wait();

  auto stage_a = [&](int s) { return sbase + s * Cfg::kStageBytes; };
  auto stage_b = [&](int s) { return stage_a(s) + Cfg::kABytes; };
  auto stage_lo = [&](int s) { return stage_b(s) + Cfg::kBBytes; };

  // Loader thread t owns output channel c = t % BN and the k range
  // [kq * KPT, kq * KPT + KPT) of every k-block.
  constexpr int KPT = 32 * BN / kSkLoaders;
  const int my_c = tid % BN;
  const int my_k0 = (tid / BN) * KPT;
  float db_acc = 0.f;

  if (warp < kSkLoaderWarps) {
    const bool split = args.split != 0;
#pragma unroll 1
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      if (!mbar_wait(tfull0 + s * 8, (i / S) & 1)) timed_out = true;
      uint8_t* b = sgen + (stage_b(s) - sbase);
      uint8_t* lo = sgen + (stage_lo(s) - sbase);
#pragma unroll
      for (int j = 0; j < KPT; ++j) {
        const uint32_t off = mnmajor_off(my_c, my_k0 + j);
        float* pb = reinterpret_cast<float*>(b + off);
        const float v = *pb;
        db_acc += v;
        if (split)
          *reinterpret_cast<float*>(lo + off) = tf32_low(v);
        else
          *pb = tf32_round(v);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(ready0 + s * 8);
    }
  } else if (warp == kSkProducerWarp) {
    if (lane == 0) {
      constexpr uint32_t bytes = Cfg::kABytes + Cfg::kBBytes;
#pragma unroll 1
      for (int j = 0; j < nk; ++j) {
        const int st = j % S;
        if (j >= S && !mbar_wait(empty0 + st * 8, ((j - S) / S) & 1)) timed_out = true;
        const int k0 = (kb0 + j) * 32;
        mbar_arrive_expect_tx(tfull0 + st * 8, bytes);
        tma_windows_mn<MT * 128>(&args.tma_a, args.a, stage_a(st), k0, tfull0 + st * 8);
#pragma unroll
        for (int g = 0; g < BN / 32; ++g)
          tma_load_2d(stage_b(st) + g * 4096, &args.tma_b, g * 32, k0, tfull0 + st * 8);
      }
    }
  } else if (lane == 0) {
    // MN-major operands (SWIZZLE_128B_BASE32B): 32-row groups 4096 B apart,
    // 4-k line groups 512 B apart; one MMA covers 8 k (1 KB).
    const uint32_t idesc = idesc_tf32(128, BN, true, true);
    const uint64_t da = umma_desc(stage_a(0), 4096u, 512u, kLayoutSw128Base32);
    const uint64_t db = umma_desc(stage_b(0), 4096u, 512u, kLayoutSw128Base32);
    const uint64_t dlo = umma_desc(stage_lo(0), 4096u, 512u, kLayoutSw128Base32);
    const bool split = args.split != 0;
#pragma unroll 1
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      if (!mbar_wait(ready0 + s * 8, (i / S) & 1)) timed_out = true;
      tc_fence_after();
      const uint64_t so = static_cast<uint64_t>(s) * (Cfg::kStageBytes >> 4);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint64_t kso = so + ks * (1024 >> 4);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const uint64_t ad = da + kso + mt * (16384 >> 4);
          const uint32_t acc = tmem + mt * BN;
          umma_tf32(acc, ad, db + kso, idesc, (i > 0 || ks > 0) ? 1u : 0u);
          if (split) umma_tf32(acc, ad, dlo + kso, idesc, 1u);
        }
      }
      umma_commit(empty0 + s * 8);
    }
    umma_commit(accum_bar);
  }

  // ---- epilogue: this CTA's partial D and column sums ----
  if (warp < kSkLoaderWarps) {
    if (nk > 0) {
      if (!mbar_wait(accum_bar, 0)) timed_out = true;
      tc_fence_after();
    }
    const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float* part = args.partial + static_cast<long long>(z) * (MT * 128) * BN;
#pragma unroll 1
    for (int mt = 0; mt < MT; ++mt) {
      const int row = mt * 128 + warp * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BN; c += 8) {
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (nk > 0) tmem_ld8(trow + mt * BN + c, v);
        float4* dst = reinterpret_cast<float4*>(part + static_cast<long long>(row) * BN + c);
        dst[0] = make_float4(v[0], v[1], v[2], v[3]);
        dst[1] = make_float4(v[4], v[5], v[6], v[7]);
      }
    }
  }
  // Column sums: KPT-wide k slices combined in slice order.
  if (warp < kSkLoaderWarps) {
    s_cols[tid / BN][my_c] = db_acc;
    asm volatile("bar.sync 1, %0;" ::"n"(kSkLoaders) : "memory");
    if (tid < BN) {
      float t = 0.f;
#pragma unroll
      for (int sl = 0; sl < SLICES; ++sl) t += s_cols[sl][tid];
      args.partial_db[static_cast<long long>(z) * BN + tid] = t;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kSkMmaWarp) tmem_dealloc(tmem, Cfg::kTmemCols);
  if (timed_out) record_error(args.status, kErrWaitTimeout);
}

// dW[c][r] (=|+=) alpha * sum_z partial[z][r][c] and db[c] (=|+=)
// sum_z partial_db[z][c], z in order. A block takes 32 consecutive (r, c)
// elements; its 8 warps sum 8 contiguous ranges of z, and the first warp
// adds the 8 range sums in order.
__global__ void __launch_bounds__(256) wgrad_sk_reduce_kernel(
    const float* __restrict__ partial, const float* __restrict__ partial_db, int ctas, int rows_pad,
    int m, int n, float alpha, float* __restrict__ dw, int accumulate, float* __restrict__ db,
    int accumulate_db) {
  pdl_trigger();
  pdl_wait();
  __shared__ float s_sum[8][32];
  const int j = threadIdx.x & 31, qz = threadIdx.x >> 5;
  const long long groups = (static_cast<long long>(m) * n + 31) / 32;
  const bool bias = blockIdx.x >= groups;
  const long long e = (bias ? (blockIdx.x - groups) : blockIdx.x) * 32ll + j;
  const long long total = bias ? n : static_cast<long long>(m) * n;
  const int per = (ctas + 7) / 8;
  const int z0 = qz * per, z1 = min(ctas, z0 + per);
  float t = 0.f;
  if (e < total) {
    if (bias) {
#pragma unroll 4
      for (int zz = z0; zz < z1; ++zz) t += partial_db[static_cast<long long>(zz) * n + e];
    } else {
      // Each CTA's D is [row][col]: element e is (r, c) = (e / n, e % n).
      const long long stride = static_cast<long long>(rows_pad) * n;
#pragma unroll 4
      for (int zz = z0; zz < z1; ++zz) t += partial[zz * stride + e];
    }
  }
  s_sum[qz][j] = t;
  __syncthreads();
  if (qz == 0 && e < total) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += s_sum[k][j];
    if (bias) {
      if (db != nullptr) db[e] = accumulate_db ? db[e] + s : s;
    } else {
      const long long r = e / n, c = e % n;
      float* o = dw + c * m + r;  // dW is [cout][taps x channels]
      const float v = alpha * s;
      *o = accumulate ? *o + v : v;
    }
  }
}

template <int MT, int BN>
cudaError_t launch_sk(const WgradSkArgs& a, cudaStream_t st) {
  using Cfg = SkCfg<MT, BN>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(wgrad_sk_kernel<MT, BN>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               Cfg::kSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  return launch_pdl(wgrad_sk_kernel<MT, BN>, dim3(a.ctas), dim3(kSkThreads), Cfg::kSmem, st, a);
}

int sm_count() {
  static int counts[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int c = 0;
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0)
      c = 148;
    counts[dev] = c;
  }
  return counts[dev];
}

int pick_mt(int m) { return m <= 128 ? 1 : m <= 256 ? 2 : 0; }

int sk_ctas(const ttrl_conv_geom* g) {
  const long long pixels = static_cast<long long>(g->n) * g->oh * g->ow;
  const int kblocks = static_cast<int>((pixels + 31) / 32);
  int ctas = sm_count();
  if (kblocks < 2 * ctas) ctas = (kblocks + 1) / 2;
  return ctas < 1 ? 1 : ctas;
}

}  // namespace

bool wgrad_sk_geometry(const ttrl_conv_geom* g) {
  if (!(g->flags & TTRL_CONV_INPUT_EXACT)) return false;  // the windows need no split
  if (g->c % 32 != 0 || (g->cout != 32 && g->cout != 64)) return false;
  if (g->kh != g->kw || pick_mt(g->kh * g->kw * g->c) == 0) return false;
  const long long pixels = static_cast<long long>(g->n) * g->oh * g->ow;
  return pixels >= 64 && pixels < (1ll << 31);
}

bool wgrad_sk_applies(const ttrl_conv_geom* g, const float* x, const float* dy) {
  const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dy);
  return wgrad_sk_geometry(g) && (al & 15u) == 0;
}

size_t wgrad_sk_ws(const ttrl_conv_geom* g) {
  const int mt = pick_mt(g->kh * g->kw * g->c);
  const size_t ctas = static_cast<size_t>(sk_ctas(g));
  return kCounterBytes + ctas * (static_cast<size_t>(mt) * 128 + 1) * g->cout * sizeof(float);
}

int wgrad_sk_run(const float* x, const float* dy, float* dw, float* db, const ttrl_conv_geom* g,
                 float alpha, int accumulate, int accumulate_db, int precision, float* ws,
                 size_t wsb, int* status, cudaStream_t st) {
  const int m = g->kh * g->kw * g->c;
  const int mt = pick_mt(m);
  const size_t need = wgrad_sk_ws(g);
  if (ws == nullptr || wsb < need)
    return set_error(TTRL_EWORKSPACE, "conv_wgrad: needs %zu bytes of workspace, got %zu", need,
                     wsb);
  WgradSkArgs a;
  std::memset(&a, 0, sizeof(a));
  ttrl_operand in;
  std::memset(&in, 0, sizeof(in));
  in.ptr = x;
  in.kind = TTRL_OPND_CONV_WGRAD;
  in.rows = m;
  in.kdim = g->n * g->oh * g->ow;
  in.flags = TTRL_OPND_EXACT_TF32;
  in.n = g->n;
  in.h = g->h;
  in.w = g->w;
  in.c = g->c;
  in.kh = g->kh;
  in.kw = g->kw;
  in.stride = g->stride;
  in.pad = g->pad;
  in.oh = g->oh;
  in.ow = g->ow;
  int rc = gemm_resolve_operand(in, 0, a.a);
  if (rc) return rc;
  if (!gemm_im2col_map(a.a, &a.tma_a))
    return set_error(TTRL_EUNSUPPORTED, "conv_wgrad: no TMA im2col map for the windows");
  ttrl_operand bo;
  std::memset(&bo, 0, sizeof(bo));
  bo.ptr = dy;
  bo.kind = TTRL_OPND_DENSE;
  bo.rows = g->cout;
  bo.kdim = in.kdim;
  bo.rs = 1;
  bo.ks = g->cout;
  DevOperand ob;
  if ((rc = gemm_resolve_operand(bo, 0, ob))) return rc;
  if (!gemm_tile_map(ob, g->cout, &a.tma_b))
    return set_error(TTRL_EUNSUPPORTED, "conv_wgrad: no TMA map for dY");
  a.kblocks = (in.kdim + 31) / 32;
  a.ctas = sk_ctas(g);
  a.split = precision == TTRL_PREC_TF32X3 ? 1 : 0;
  a.partial = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + kCounterBytes);
  a.partial_db = a.partial + static_cast<size_t>(a.ctas) * mt * 128 * g->cout;
  a.status = status;
  cudaError_t e;
  if (mt == 1)
    e = g->cout == 32 ? launch_sk<1, 32>(a, st) : launch_sk<1, 64>(a, st);
  else
    e = g->cout == 32 ? launch_sk<2, 32>(a, st) : launch_sk<2, 64>(a, st);
  note_launch();
  if (e != cudaSuccess) return set_cuda_error("conv_wgrad stream-K launch", e);
  const long long groups = (static_cast<long long>(m) * g->cout + 31) / 32 + (g->cout + 31) / 32;
  e = launch_pdl(wgrad_sk_reduce_kernel, dim3(static_cast<unsigned>(groups)), dim3(256), 0, st,
                 a.partial, a.partial_db, a.ctas, mt * 128, m, g->cout, alpha, dw, accumulate, db,
                 accumulate_db);
  note_launch();
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("conv_wgrad stream-K reduce launch", e);
}

}  // namespace ttrl
