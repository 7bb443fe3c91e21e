// Prioritized replay on the device (ttrl/buffers/sampling.py:111-240,
// ttrl/algos/offpolicy.py:136-145): the priority table lives in HBM as
// float64 [lanes][columns] holding (p + eps)^alpha, so a DQN update's |TD|
// errors are written back by the device straight from the loss kernel's
// output, with no host read in between.
//
// per_update_kernel: table[lane][col] = (|td| + eps)^alpha for one batch,
// where a (lane, col) pair drawn twice takes its LAST value (numpy's fancy
// assignment), and max_priority = max(max_priority, max |td|). With
// `from_max` set it writes (max_priority + eps)^alpha instead: a freshly
// written column's priority (on_write). A non-finite |td| records 1003 and
// leaves the table as it was.
// per_cdf_kernel: each lane's run (window positions 0 .. count-1, oldest
// first, column (start + p) % columns) summed sequentially in float64, the
// order of numpy's cumsum; the last value is the lane's total.
// per_draw_kernel: one sample per thread, the reference's searchsorted draw
// within its lane: target = u * cdf[count-1], position = first p with
// cdf[p] > target (side="right"), clipped to count-1.
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace ttrl {

constexpr int kPerThreads = 1024;
constexpr int kErrNonFinite = 1003;

__global__ void __launch_bounds__(kPerThreads) per_update_kernel(
    double* __restrict__ table, int columns, const int32_t* __restrict__ lanes,
    const int32_t* __restrict__ cols, const float* __restrict__ td, int batch, double alpha,
    double eps, double* __restrict__ max_priority, int from_max, int* status) {
  pdl_trigger();
  pdl_wait();
  __shared__ double red[kPerThreads];
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  double local_max = 0.0;
  for (int b = threadIdx.x; b < batch; b += kPerThreads) {
    const double p = from_max ? *max_priority : fabs(static_cast<double>(td[b]));
    if (!isfinite(p)) {
      bad = 1;
    } else {
      local_max = fmax(local_max, p);
    }
  }
  red[threadIdx.x] = local_max;
  __syncthreads();
  for (int w = kPerThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] = fmax(red[threadIdx.x], red[threadIdx.x + w]);
    __syncthreads();
  }
  if (bad) {
    if (threadIdx.x == 0) record_error(status, kErrNonFinite);
    return;
  }
  const double base = from_max ? *max_priority : 0.0;
  for (int b = threadIdx.x; b < batch; b += kPerThreads) {
    const int l = lanes[b], c = cols[b];
    bool later = false;
    for (int q = b + 1; q < batch && !later; ++q) later = lanes[q] == l && cols[q] == c;
    if (later) continue;
    const double p = from_max ? base : fabs(static_cast<double>(td[b]));
    table[static_cast<long long>(l) * columns + c] = pow(p + eps, alpha);
  }
  __syncthreads();
  if (threadIdx.x == 0 && !from_max) *max_priority = fmax(*max_priority, red[0]);
}

__global__ void per_cdf_kernel(const double* __restrict__ table, int n_lanes, int columns,
                               const int32_t* __restrict__ counts,
                               const int32_t* __restrict__ start, double* __restrict__ cdf,
                               double* __restrict__ totals) {
  pdl_trigger();
  pdl_wait();
  const int l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l >= n_lanes) return;
  const int n = counts[l];
  const double* row = table + static_cast<long long>(l) * columns;
  double* out = cdf + static_cast<long long>(l) * columns;
  double s = 0.0;
  int c = start[l] % columns;
  for (int p = 0; p < n; ++p) {
    s += row[c];
    out[p] = s;
    if (++c == columns) c = 0;
  }
  totals[l] = s;
}

__global__ void per_draw_kernel(const double* __restrict__ cdf, const double* __restrict__ table,
                                int columns, const int32_t* __restrict__ counts,
                                const int32_t* __restrict__ start,
                                const int32_t* __restrict__ lane_of,
                                const double* __restrict__ uniforms, int batch,
                                int32_t* __restrict__ positions, int32_t* __restrict__ out_cols,
                                double* __restrict__ picked) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const int l = lane_of[b];
  const int n = counts[l];
  const double* row = cdf + static_cast<long long>(l) * columns;
  const double target = uniforms[b] * row[n - 1];
  int lo = 0, hi = n;  // first p in [0, n) with row[p] > target, else n
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (row[mid] > target) {
      hi = mid;
    } else {
      lo = mid + 1;
    }
  }
  const int p = lo < n - 1 ? lo : n - 1;
  const int col = static_cast<int>((static_cast<long long>(start[l]) + p) % columns);
  positions[b] = p;
  out_cols[b] = col;
  picked[b] = table[static_cast<long long>(l) * columns + col];
}

int per_update(double* table, int columns, const int32_t* lanes, const int32_t* cols,
               const float* td, int batch, double alpha, double eps, double* max_priority,
               int from_max, int* status, cudaStream_t st) {
  if (batch <= 0 || columns <= 0) return set_error(TTRL_EINVAL, "per_update: empty batch");
  if (!table || !lanes || !cols || !max_priority || (!from_max && !td))
    return set_error(TTRL_EINVAL, "per_update: null pointer");
  const cudaError_t le = launch_pdl(per_update_kernel, dim3(1), dim3(kPerThreads), 0, st, table,
                                    columns, lanes, cols, td, batch, alpha, eps, max_priority,
                                    from_max, status);
  note_launch();
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("per_update launch", e);
}

int per_cdf(const double* table, int n_lanes, int columns, const int32_t* counts,
            const int32_t* start, double* cdf, double* totals, cudaStream_t st) {
  if (n_lanes <= 0 || columns <= 0) return set_error(TTRL_EINVAL, "per_cdf: empty table");
  if (!table || !counts || !start || !cdf || !totals)
    return set_error(TTRL_EINVAL, "per_cdf: null pointer");
  const cudaError_t le = launch_pdl(per_cdf_kernel, dim3((n_lanes + 31) / 32), dim3(32), 0, st,
                                    table, n_lanes, columns, counts, start, cdf, totals);
  note_launch();
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("per_cdf launch", e);
}

int per_draw(const double* cdf, const double* table, int columns, const int32_t* counts,
             const int32_t* start, const int32_t* lane_of, const double* uniforms, int batch,
             int32_t* positions, int32_t* out_cols, double* picked, cudaStream_t st) {
  if (batch <= 0 || columns <= 0) return set_error(TTRL_EINVAL, "per_draw: empty batch");
  if (!cdf || !table || !counts || !start || !lane_of || !uniforms || !positions || !out_cols ||
      !picked)
    return set_error(TTRL_EINVAL, "per_draw: null pointer");
  const cudaError_t le = launch_pdl(per_draw_kernel, dim3((batch + 127) / 128), dim3(128), 0, st,
                                    cdf, table, columns, counts, start, lane_of, uniforms, batch,
                                    positions, out_cols, picked);
  note_launch();
  const cudaError_t e = le != cudaSuccess ? le : cudaGetLastError();
  return e == cudaSuccess ? TTRL_OK : set_cuda_error("per_draw launch", e);
}

}  // namespace ttrl

using namespace ttrl;

extern "C" {

int ttrl_per_update(double* table, int columns, const int32_t* lanes, const int32_t* cols,
                    const float* td_abs, int batch, double alpha, double eps,
                    double* max_priority, int from_max, int* status, ttrl_stream_t stream) {
  return per_update(table, columns, lanes, cols, td_abs, batch, alpha, eps, max_priority,
                    from_max, status, static_cast<cudaStream_t>(stream));
}

int ttrl_per_cdf(const double* table, int n_lanes, int columns, const int32_t* counts,
                 const int32_t* start, double* cdf, double* totals, ttrl_stream_t stream) {
  return per_cdf(table, n_lanes, columns, counts, start, cdf, totals,
                 static_cast<cudaStream_t>(stream));
}

int ttrl_per_draw(const double* cdf, const double* table, int columns, const int32_t* counts,
                  const int32_t* start, const int32_t* lane_of, const double* uniforms, int batch,
                  int32_t* positions, int32_t* cols, double* picked, ttrl_stream_t stream) {
  return per_draw(cdf, table, columns, counts, start, lane_of, uniforms, batch, positions, cols,
                  picked, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
