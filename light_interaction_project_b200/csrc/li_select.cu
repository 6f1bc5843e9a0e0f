// Block selection: pooled-score GEMM, protection bias, top-k, sorted emit.
//
// One CTA (4 warps) handles R <= 4 query rows of one (b, h). The query rows
// and then the key rows, 32 at a time, are staged in shared memory as doubles
// with coalesced 16-byte loads ('cosine' normalises them there; the pipeline
// normalises pools once with li_normalize_rows and selects with the plain dot
// product instead). Warp r forms the dot products of query row r with the 32
// staged key rows, one per lane.
// Dot products and squared norms are exact-product fp64 sums (four interleaved
// partial sums over d, combined in order), rounded once to fp32 and then to
// the dtype; scalar multiplies/adds are single fp32 operations rounded to the
// dtype (torch's opmath rule). The ranking value is mapped to torch's radix
// key and kept in shared memory.
//
// Warp r then selects row r's top k: a 64-bit composite key
// (radix_key << idx_bits) | (2^idx_bits - 1 - j) is unique per column and
// orders equal scores lowest index first. A bitwise search finds the k-th
// largest composite (count of keys >= candidate via ballots), and one pass in
// ascending j emits every column at or above it with a ballot prefix sum —
// already sorted ascending, so no sort is needed.
#include <cmath>
#include <cstring>
#include <mutex>

#include "li_common.cuh"

namespace li {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxD = 256;
constexpr size_t kSmemBudget = 160 * 1024;

struct SelArgs {
  const uint8_t* qp; int64_t q_b, q_h, q_n;
  const uint8_t* kp; int64_t k_b, k_h, k_n;
  const float* bias; int64_t x_b, x_h, x_q, x_k;
  int32_t* idx; int64_t i_b, i_h, i_q, i_s;
  int32_t* cnt; int64_t c_b, c_h, c_q;
  float* rank; int64_t r_b, r_h, r_q, r_k;
  int32_t H, D, Nq, Nk, dtype, metric, mode;
  int32_t n_prot;          // decode
  int32_t g_nh, g_nw;      // bidir key grid (Nh, Nw)
  int32_t q_off;           // bidir
  int32_t k_budget, ntxt, R, idx_bits, key_bits;
  float scale;             // fp32(1/sqrt(D)) for scaled_dot_product
  float big;               // decode: fp32(1e6); bidir: dtype(fp32(1)*fp32(1e6))
  float eps;               // dtype(fp32(1e-12))
};

__device__ __forceinline__ uint32_t radix_key(float v, int dt) {
  if (v != v) return dt == LI_DTYPE_FP32 ? 0xFFFFFFFFu : 0xFFFFu;  // NaN ranks highest
  if (dt == LI_DTYPE_FP32) {
    const uint32_t x = __float_as_uint(v);
    return x ^ ((x & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
  }
  uint32_t x;
  if (dt == LI_DTYPE_BF16) x = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  else x = __half_as_ushort(__float2half_rn(v));
  return x ^ ((x & 0x8000u) ? 0xFFFFu : 0x8000u);
}

// Four interleaved fp64 partial sums of exact products, combined in order —
// the summation order the CPU oracle restates.
template <typename T>
__device__ __forceinline__ double dot4(const T* x, const T* y, int D) {
  double p0 = 0.0, p1 = 0.0, p2 = 0.0, p3 = 0.0;
  for (int d = 0; d < D; d += 4) {
    p0 = fma((double)x[d], (double)y[d], p0);
    p1 = fma((double)x[d + 1], (double)y[d + 1], p1);
    p2 = fma((double)x[d + 2], (double)y[d + 2], p2);
    p3 = fma((double)x[d + 3], (double)y[d + 3], p3);
  }
  return ((p0 + p1) + p2) + p3;
}

// 16-byte chunk of a pooled row -> doubles (exact widening).
__device__ __forceinline__ void widen_chunk(const uint4& v, int dt, double* dst) {
  const int epc = dt == LI_DTYPE_FP32 ? 4 : 8;
#pragma unroll
  for (int e = 0; e < 8; ++e)
    if (e < epc) dst[e] = chunk_elem_f64(v, e, dt);
}

constexpr int kChunkRows = 32;

// Normalisation of F.normalize on a staged row (dtype values held as doubles).
__device__ __forceinline__ void normalize_row(double* x, int D, int dt, float eps) {
  const float den = fmaxf(round_dt(__fsqrt_rn(__double2float_rn(dot4(x, x, D))), dt), eps);
  for (int d = 0; d < D; ++d) x[d] = (double)round_dt(__fdiv_rn((float)x[d], den), dt);
}

template <int R>
__global__ void __launch_bounds__(kThreads) select_kernel(const SelArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int pitch = a.D + 1;                                    // doubles; odd pitch spreads banks
  double* qs = reinterpret_cast<double*>(smem);                 // [R][pitch]
  double* ks = qs + R * pitch;                                  // [kChunkRows][pitch]
  uint32_t* keys = reinterpret_cast<uint32_t*>(ks + kChunkRows * pitch);  // [R][Nk]
  const int bh = blockIdx.y;
  const int b = bh / a.H, h = bh % a.H;
  const int q0 = blockIdx.x * R;
  const int nrows = min(R, a.Nq - q0);
  const int tid = threadIdx.x;
  const int es = a.dtype == LI_DTYPE_FP32 ? 4 : 2;
  const int epc = 16 / es;
  const int CH = a.D / epc;
  const bool cosine = a.metric == LI_METRIC_COSINE;

  // Query rows (normalised for 'cosine').
  for (int i = tid; i < R * CH; i += kThreads) {
    const int r = i / CH, c = i % CH;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nrows)
      v = __ldg(reinterpret_cast<const uint4*>(a.qp + (b * a.q_b + h * a.q_h + (int64_t)(q0 + r) * a.q_n) * es) + c);
    widen_chunk(v, a.dtype, qs + r * pitch + c * epc);
  }
  __syncthreads();
  if (cosine && tid < nrows) normalize_row(qs + tid * pitch, a.D, a.dtype, a.eps);

  const uint8_t* kbase = a.kp + (b * a.k_b + h * a.k_h) * es;
  const int warp = tid / 32, lane = tid % 32;
  for (int c0 = 0; c0 < a.Nk; c0 += kChunkRows) {
    __syncthreads();
    for (int i = tid; i < kChunkRows * CH; i += kThreads) {
      const int r = i / CH, c = i % CH;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (c0 + r < a.Nk) v = __ldg(reinterpret_cast<const uint4*>(kbase + (int64_t)(c0 + r) * a.k_n * es) + c);
      widen_chunk(v, a.dtype, ks + r * pitch + c * epc);
    }
    __syncthreads();
    if (cosine) {
      if (tid < kChunkRows) normalize_row(ks + tid * pitch, a.D, a.dtype, a.eps);
      __syncthreads();
    }
    // Warp w forms the dot products of its query rows with the 32 staged key rows.
    for (int r = warp; r < nrows; r += kWarps) {
      const int j = c0 + lane;
      if (j >= a.Nk) continue;
      const int qi = q0 + r;
      float s = round_dt(__double2float_rn(dot4(qs + r * pitch, ks + lane * pitch, a.D)), a.dtype);
      if (a.metric == LI_METRIC_SCALED_DOT) s = round_dt(__fmul_rn(s, a.scale), a.dtype);
      if (a.bias)
        s = round_dt(__fadd_rn(s, a.bias[b * a.x_b + h * a.x_h + qi * a.x_q + (int64_t)j * a.x_k]), a.dtype);
      if (a.mode == LI_SELECT_DECODE) {
        if (j >= a.Nk - a.n_prot) s = round_dt(__fadd_rn(s, a.big), a.dtype);
      } else {
        const int gq = qi + a.q_off;
        const int hw = a.g_nh * a.g_nw;
        const int tq = gq / hw, hq = (gq % hw) / a.g_nw, wq = gq % a.g_nw;
        const int tk = j / hw, hk = (j % hw) / a.g_nw, wk = j % a.g_nw;
        const int dist = abs(tq - tk) + abs(hq - hk) + abs(wq - wk);
        s = round_dt(__fadd_rn(s, dist <= 1 ? a.big : 0.0f), a.dtype);
      }
      keys[r * a.Nk + j] = radix_key(s, a.dtype);
      if (a.rank) a.rank[b * a.r_b + h * a.r_h + qi * a.r_q + (int64_t)j * a.r_k] = s;
    }
  }
  __syncthreads();

  for (int r = warp; r < nrows; r += kWarps) {
    const int qi = q0 + r;
    const uint32_t* rk = keys + r * a.Nk;
    const uint64_t low_mask = (1ull << a.idx_bits) - 1ull;
    const int k = a.k_budget;
    uint64_t thr = 0;
    if (k > 0 && k < a.Nk) {
      for (int bit = a.key_bits + a.idx_bits - 1; bit >= 0; --bit) {
        const uint64_t cand = thr | (1ull << bit);
        int c = 0;
        for (int j = lane; j < a.Nk; j += 32) {
          const uint64_t comp = ((uint64_t)rk[j] << a.idx_bits) | (low_mask - (uint64_t)j);
          c += comp >= cand;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
        if (c >= k) thr = cand;
      }
    }
    int32_t* out = a.idx + b * a.i_b + h * a.i_h + (int64_t)qi * a.i_q;
    for (int t = lane; t < a.ntxt; t += 32) out[(int64_t)t * a.i_s] = t;
    int pos = 0;
    if (k > 0) {
      for (int base = 0; base < a.Nk; base += 32) {
        const int j = base + lane;
        bool sel = false;
        if (j < a.Nk) {
          const uint64_t comp = ((uint64_t)rk[j] << a.idx_bits) | (low_mask - (uint64_t)j);
          sel = (k >= a.Nk) || comp >= thr;
        }
        const unsigned m = __ballot_sync(0xFFFFFFFFu, sel);
        if (sel) out[(int64_t)(a.ntxt + pos + __popc(m & ((1u << lane) - 1u))) * a.i_s] = j + a.ntxt;
        pos += __popc(m);
      }
    }
    if (lane == 0) a.cnt[b * a.c_b + h * a.c_h + (int64_t)qi * a.c_q] = a.ntxt + k;
  }
}

// ---------------------------------------------------------------------------
// Two-kernel form (with a workspace): scores over a (row group, key chunk, b*h)
// grid, then top-k per row. Same arithmetic as select_kernel.
// ---------------------------------------------------------------------------
constexpr int kScoreRows = 8;    // query rows per CTA (two groups of four)
constexpr int kScoreKeys = 64;   // key rows per CTA

__device__ __forceinline__ float finish_score(const SelArgs& a, double acc, int b, int h, int qi, int j) {
  float s = round_dt(__double2float_rn(acc), a.dtype);
  if (a.metric == LI_METRIC_SCALED_DOT) s = round_dt(__fmul_rn(s, a.scale), a.dtype);
  if (a.bias) s = round_dt(__fadd_rn(s, a.bias[b * a.x_b + h * a.x_h + qi * a.x_q + (int64_t)j * a.x_k]), a.dtype);
  if (a.mode == LI_SELECT_DECODE) {
    if (j >= a.Nk - a.n_prot) s = round_dt(__fadd_rn(s, a.big), a.dtype);
  } else {
    const int gq = qi + a.q_off;
    const int hw = a.g_nh * a.g_nw;
    const int tq = gq / hw, hq = (gq % hw) / a.g_nw, wq = gq % a.g_nw;
    const int tk = j / hw, hk = (j % hw) / a.g_nw, wk = j % a.g_nw;
    const int dist = abs(tq - tk) + abs(hq - hk) + abs(wq - wk);
    s = round_dt(__fadd_rn(s, dist <= 1 ? a.big : 0.0f), a.dtype);
  }
  return s;
}

__global__ void __launch_bounds__(128) score_kernel(const SelArgs a, uint32_t* __restrict__ keys) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int pitch = a.D + 1;
  double* qs = reinterpret_cast<double*>(smem);            // [kScoreRows][pitch]
  double* ks = qs + kScoreRows * pitch;                    // [kScoreKeys][pitch]
  const int bh = blockIdx.z, b = bh / a.H, h = bh % a.H;
  const int q0 = blockIdx.x * kScoreRows, j0 = blockIdx.y * kScoreKeys;
  const int nrows = min(kScoreRows, a.Nq - q0), nkeys = min(kScoreKeys, a.Nk - j0);
  const int tid = threadIdx.x;
  const int es = a.dtype == LI_DTYPE_FP32 ? 4 : 2, epc = 16 / es, CH = a.D / epc;
  for (int i = tid; i < kScoreRows * CH; i += 128) {
    const int r = i / CH, c = i % CH;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nrows) v = __ldg(reinterpret_cast<const uint4*>(a.qp + (b * a.q_b + h * a.q_h + (int64_t)(q0 + r) * a.q_n) * es) + c);
    widen_chunk(v, a.dtype, qs + r * pitch + c * epc);
  }
  for (int i = tid; i < kScoreKeys * CH; i += 128) {
    const int r = i / CH, c = i % CH;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nkeys) v = __ldg(reinterpret_cast<const uint4*>(a.kp + (b * a.k_b + h * a.k_h + (int64_t)(j0 + r) * a.k_n) * es) + c);
    widen_chunk(v, a.dtype, ks + r * pitch + c * epc);
  }
  __syncthreads();
  if (a.metric == LI_METRIC_COSINE) {
    if (tid < nrows) normalize_row(qs + tid * pitch, a.D, a.dtype, a.eps);
    if (tid >= 64 && tid - 64 < nkeys) normalize_row(ks + (tid - 64) * pitch, a.D, a.dtype, a.eps);
    __syncthreads();
  }
  // Thread (g, jj): key jj against query rows 4g..4g+3, four partial sums each.
  const int jj = tid % kScoreKeys, g = tid / kScoreKeys;
  if (jj >= nkeys) return;
  const double* kr = ks + jj * pitch;
  const double* q0r = qs + (4 * g) * pitch;
  double acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int u = 0; u < 4; ++u) acc[r][u] = 0.0;
  for (int d = 0; d < a.D; d += 4) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const double kv = kr[d + u];
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[r][u] = fma(q0r[r * pitch + d + u], kv, acc[r][u]);
    }
  }
  const int j = j0 + jj;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int lr = 4 * g + r;
    if (lr >= nrows) break;
    const int qi = q0 + lr;
    const double dot = ((acc[r][0] + acc[r][1]) + acc[r][2]) + acc[r][3];
    const float s = finish_score(a, dot, b, h, qi, j);
    keys[((int64_t)bh * a.Nq + qi) * a.Nk + j] = radix_key(s, a.dtype);
    if (a.rank) a.rank[b * a.r_b + h * a.r_h + qi * a.r_q + (int64_t)j * a.r_k] = s;
  }
}

// Register-tiled scores for the dot metrics (no in-kernel normalisation): a
// CTA of 256 threads takes 16 query rows x 64M keys; thread (rg, kh, kq) forms
// rows 4rg..4rg+3 against keys 32M kh + kq + 32m (m < M), each with the four
// interleaved fp64 partial sums of the fixed order. D is staged 32 columns at
// a time; the next slice's global loads are in flight while the current one
// is used. M = 2 (128 keys) normally; M = 1 doubles the CTA count when the
// grid would otherwise fill fewer than two waves of the GPU (few heads).
constexpr int kTileRows = 16, kTileKeysMax = 128, kTileD = 32, kTileThreads = 256;
template <int DT, int M>
__global__ void __launch_bounds__(kTileThreads, 2) score_tile_kernel(const SelArgs a, uint32_t* __restrict__ keys) {
  constexpr int kTileKeys = 64 * M;
  extern __shared__ __align__(16) uint8_t smem[];
  // K rows: odd pitch, so a warp's 32 keys hit distinct bank pairs. Q rows: even
  // pitch, so a thread reads two consecutive d of a row as one 16-byte broadcast.
  constexpr int pitch = kTileD + 1, qpitch = kTileD + 2;
  double* qs = reinterpret_cast<double*>(smem);          // [kTileRows][qpitch]
  double* ks = qs + kTileRows * qpitch;                  // [kTileKeys][pitch]
  const int bh = blockIdx.z, b = bh / a.H, h = bh % a.H;
  const int q0 = blockIdx.x * kTileRows, j0 = blockIdx.y * kTileKeys;
  const int nrows = min(kTileRows, a.Nq - q0), nkeys = min(kTileKeys, a.Nk - j0);
  const int tid = threadIdx.x, warp = tid >> 5, kq = tid & 31;
  const int rg = warp >> 1, kh = warp & 1;
  constexpr int es = DT == LI_DTYPE_FP32 ? 4 : 2, epc = 16 / es, CHD = kTileD / epc;  // 16-byte chunks per slice row
  constexpr int kLoads = ((kTileRows + kTileKeys) * CHD + kTileThreads - 1) / kTileThreads;
  const uint8_t* qbase = a.qp + (b * a.q_b + h * a.q_h) * es;
  const uint8_t* kbase = a.kp + (b * a.k_b + h * a.k_h) * es;
  uint4 pre[kLoads];
  auto fetch = [&](int dc) {
#pragma unroll
    for (int l = 0; l < kLoads; ++l) {
      const int i = tid + l * kTileThreads;
      const int r = i / CHD, c = i % CHD;
      pre[l] = make_uint4(0, 0, 0, 0);
      if (r < kTileRows) {
        if (r < nrows) pre[l] = __ldg(reinterpret_cast<const uint4*>(qbase + ((int64_t)(q0 + r) * a.q_n + dc) * es) + c);
      } else if (r < kTileRows + kTileKeys) {
        const int kr = r - kTileRows;
        if (kr < nkeys) pre[l] = __ldg(reinterpret_cast<const uint4*>(kbase + ((int64_t)(j0 + kr) * a.k_n + dc) * es) + c);
      }
    }
  };
  auto stage = [&]() {
#pragma unroll
    for (int l = 0; l < kLoads; ++l) {
      const int i = tid + l * kTileThreads;
      const int r = i / CHD, c = i % CHD;
      if (r >= kTileRows + kTileKeys) continue;
      double* dst = (r < kTileRows ? qs + r * qpitch : ks + (r - kTileRows) * pitch) + c * epc;
#pragma unroll
      for (int e = 0; e < epc; ++e) dst[e] = (double)chunk_elem(pre[l], e, DT);
    }
  };
  double acc[4][M][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[r][m][u] = 0.0;
  fetch(0);
  stage();
  __syncthreads();
  for (int dc = 0; dc < a.D; dc += kTileD) {
    const bool more = dc + kTileD < a.D;
    if (more) fetch(dc + kTileD);
#pragma unroll 2
    for (int d = 0; d < kTileD; d += 4) {
#pragma unroll
      for (int u2 = 0; u2 < 4; u2 += 2) {
        double2 q2[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) q2[r] = *reinterpret_cast<const double2*>(qs + (4 * rg + r) * qpitch + d + u2);
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int u = u2 + h2;
          double kv[M];
#pragma unroll
          for (int m = 0; m < M; ++m) kv[m] = ks[(32 * M * kh + kq + 32 * m) * pitch + d + u];
#pragma unroll
          for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int m = 0; m < M; ++m) acc[r][m][u] = fma(h2 ? q2[r].y : q2[r].x, kv[m], acc[r][m][u]);
        }
      }
    }
    if (more) {
      __syncthreads();
      stage();
      __syncthreads();
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int lr = 4 * rg + r;
    if (lr >= nrows) break;
    const int qi = q0 + lr;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const int kr = 32 * M * kh + kq + 32 * m;
      if (kr >= nkeys) continue;
      const int j = j0 + kr;
      const double dot = ((acc[r][m][0] + acc[r][m][1]) + acc[r][m][2]) + acc[r][m][3];
      const float sc = finish_score(a, dot, b, h, qi, j);
      keys[((int64_t)bh * a.Nq + qi) * a.Nk + j] = radix_key(sc, DT);
      if (a.rank) a.rank[b * a.r_b + h * a.r_h + qi * a.r_q + (int64_t)j * a.r_k] = sc;
    }
  }
}

// One CTA of 256 threads per query row: top-k of the precomputed radix keys,
// emitted sorted. An 8-bit radix select finds the k-th largest key T (key_bits / 8
// histogram passes over the row in shared memory; thread t owns digit 255 - t
// and a block scan of the 256 counts finds the digit holding rank k); one pass
// in ascending j then emits every key above T and the lowest-index keys equal
// to T until k are taken — the order of the composite key
// (radix_key << idx_bits) | (2^idx_bits - 1 - j), ties to the lowest index.
// Thread t emits the contiguous keys [t*per, (t+1)*per): block scans of its
// tie and selection counts give each thread its ties already taken and its
// output position.
constexpr int kTopkThreads = 256;

// Exclusive block scan of one value per thread (kTopkThreads threads); *total is
// the block sum. scratch: 8 words, reusable when the call returns.
__device__ __forceinline__ uint32_t block_exscan(uint32_t v, uint32_t* scratch, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) scratch[warp] = inc;
  __syncthreads();
  uint32_t base = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < kTopkThreads / 32; ++w) {
    const uint32_t x = scratch[w];
    base += w < warp ? x : 0u;
    tot += x;
  }
  __syncthreads();
  *total = tot;
  return base + inc - v;
}

__global__ void __launch_bounds__(kTopkThreads) topk_kernel(const SelArgs a, const uint32_t* __restrict__ keys) {
  static_assert(kTopkThreads == 256, "one thread per radix digit");
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem);  // 256 bins
  uint32_t* scratch = hist + 256;                      // scan scratch, then the found digit
  uint32_t* rk = hist + 256 + 16;                      // the row's Nk keys
  const int t = threadIdx.x;
  const int qi = blockIdx.x, bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const uint32_t* src = keys + ((int64_t)bh * a.Nq + qi) * a.Nk;
  for (int j = t; j < a.Nk; j += kTopkThreads) rk[j] = src[j];
  __syncthreads();
  const int k = a.k_budget;
  uint32_t T = 0;  // the k-th largest key
  int ties = 0;    // keys equal to T that are taken
  if (k > 0 && k < a.Nk) {
    uint32_t prefix = 0;
    int need = k;  // rank of the k-th largest within the keys matching `prefix`
    for (int shift = a.key_bits - 8; shift >= 0; shift -= 8) {
      const uint32_t hi = shift + 8 >= 32 ? 0u : (0xFFFFFFFFu << (shift + 8));
      hist[t] = 0;
      __syncthreads();
      for (int j = t; j < a.Nk; j += kTopkThreads) {
        const uint32_t key = rk[j];
        if ((key & hi) == prefix) atomicAdd(&hist[(key >> shift) & 0xFFu], 1u);
      }
      __syncthreads();
      // Thread t owns digit 255 - t: counts of larger digits come first.
      const uint32_t c = hist[255 - t];
      uint32_t total;
      const uint32_t before = block_exscan(c, scratch, &total);
      if ((int)before < need && (int)(before + c) >= need) {
        scratch[8] = 255u - (uint32_t)t;
        scratch[9] = (uint32_t)(need - (int)before);
      }
      __syncthreads();
      prefix |= scratch[8] << shift;
      need = (int)scratch[9];
      __syncthreads();
    }
    T = prefix;
    ties = need;
  }
  int32_t* out = a.idx + b * a.i_b + h * a.i_h + (int64_t)qi * a.i_q;
  for (int x = t; x < a.ntxt; x += kTopkThreads) out[(int64_t)x * a.i_s] = x;
  if (k > 0) {
    const int per = (a.Nk + kTopkThreads - 1) / kTopkThreads;
    const int j0 = t * per < a.Nk ? t * per : a.Nk, j1 = j0 + per < a.Nk ? j0 + per : a.Nk;
    const bool all = k >= a.Nk;
    uint32_t n_eq = 0;
    for (int j = j0; j < j1; ++j) n_eq += rk[j] == T ? 1u : 0u;
    uint32_t total;
    const uint32_t eq_before = block_exscan(n_eq, scratch, &total);
    uint32_t n_sel = 0;
    {
      uint32_t e = eq_before;
      for (int j = j0; j < j1; ++j) {
        const uint32_t key = rk[j];
        const bool eq = key == T;
        n_sel += (all || key > T || (eq && (int)e < ties)) ? 1u : 0u;
        e += eq ? 1u : 0u;
      }
    }
    uint32_t pos = block_exscan(n_sel, scratch, &total);
    uint32_t e = eq_before;
    for (int j = j0; j < j1; ++j) {
      const uint32_t key = rk[j];
      const bool eq = key == T;
      if (all || key > T || (eq && (int)e < ties)) out[(int64_t)(a.ntxt + (int)pos++) * a.i_s] = j + a.ntxt;
      e += eq ? 1u : 0u;
    }
  }
  if (t == 0) a.cnt[b * a.c_b + h * a.c_h + (int64_t)qi * a.c_q] = a.ntxt + k;
}

li_status budget_of(const li_select_params* p, int64_t nq, int64_t nk, int32_t* ntxt, int32_t* kb,
                    int32_t* nprot) {
  if (!p) return fail(LI_ERR_INVALID_ARG, "params required");
  if (p->tt <= 0 || p->th <= 0 || p->tw <= 0) return fail(LI_ERR_INVALID_ARG, "bad tile_size");
  const int64_t bs = (int64_t)p->tt * p->th * p->tw;
  if (p->text_len < 0) return fail(LI_ERR_INVALID_ARG, "text_len < 0");
  *ntxt = (int32_t)((p->text_len + bs - 1) / bs);
  *nprot = 0;
  if (p->mode == LI_SELECT_DECODE) {
    int64_t n_prot = 0;
    if (p->recent_protect > 0) {
      n_prot = ((int64_t)(p->recent_protect + p->tt - 1) / p->tt) * p->grid_q[1] * p->grid_q[2];
      if (n_prot > nk) n_prot = nk;
    }
    const int64_t n_hist = nk - n_prot > 0 ? nk - n_prot : 0;
    int64_t k = n_prot + (int64_t)((double)n_hist * p->topk_ratio);
    const int64_t lo = nk > 0 ? 1 : 0;
    if (k < lo) k = lo;
    if (k > nk) k = nk;
    *kb = (int32_t)k;
    *nprot = (int32_t)n_prot;
  } else if (p->mode == LI_SELECT_BIDIR) {
    int64_t k = (int64_t)((double)nk * p->topk_ratio);
    if (k < p->min_budget) k = p->min_budget;
    if (k > nk) k = nk;
    *kb = (int32_t)k;
  } else {
    return fail(LI_ERR_INVALID_ARG, "unknown selection mode %d", p->mode);
  }
  (void)nq;
  return LI_OK;
}

li_status check_index_out(const li_index_view* o, int64_t B, int64_t H, int64_t Nq, int64_t cols) {
  if (!o || !o->indices || !o->counts) return fail(LI_ERR_INVALID_ARG, "index output required");
  if (o->shape[0] != B || o->shape[1] != H || o->shape[2] != Nq || o->shape[3] != cols)
    return fail(LI_ERR_SHAPE, "indices: expected [%lld,%lld,%lld,%lld], got [%lld,%lld,%lld,%lld]",
                (long long)B, (long long)H, (long long)Nq, (long long)cols, (long long)o->shape[0],
                (long long)o->shape[1], (long long)o->shape[2], (long long)o->shape[3]);
  return LI_OK;
}

template <int R>
li_status launch_select(const SelArgs& a, dim3 grid, size_t smem, cudaStream_t s) {
  static std::atomic<uint64_t> configured{0};
  if (li_status st = once_per_device(configured, [] {
        return cuda_status(cudaFuncSetAttribute(select_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                (int)kSmemBudget), "select_kernel smem attribute");
      })) return st;
  select_kernel<R><<<grid, kThreads, smem, s>>>(a);
  return launched("select_kernel launch");
}

}  // namespace
}  // namespace li

using namespace li;

namespace li {
namespace {
// Row-wise F.normalize of pooled rows, exactly as the selection kernel does it
// for 'cosine'. 64 rows per CTA are staged as doubles. The four interleaved
// fp64 partial sums of squares of a row go to four adjacent lanes and are
// combined in order ((p0 + p1) + p2) + p3 through shuffles; then all 256
// threads divide and store 16-byte chunks. DT is the element type.
constexpr int kNormRows = 64, kNormThreads = 256;
template <int DT>
__global__ void __launch_bounds__(kNormThreads) normalize_kernel(const uint8_t* x, int64_t x_b, int64_t x_h,
                                                                  int64_t x_n, uint8_t* y, int64_t y_b, int64_t y_h,
                                                                  int64_t y_n, int H, int N, int D, float eps) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int pitch = D + 1;
  double* rows = reinterpret_cast<double*>(smem);                       // [64][pitch]
  float* den = reinterpret_cast<float*>(rows + kNormRows * pitch);      // [64]
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int n0 = blockIdx.x * kNormRows;
  constexpr int es = DT == LI_DTYPE_FP32 ? 4 : 2, epc = 16 / es;
  const int CH = D / epc;
  for (int i = threadIdx.x; i < kNormRows * CH; i += kNormThreads) {
    const int r = i / CH, c = i % CH;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (n0 + r < N) v = __ldg(reinterpret_cast<const uint4*>(x + (b * x_b + h * x_h + (int64_t)(n0 + r) * x_n) * es) + c);
    widen_chunk(v, DT, rows + r * pitch + c * epc);
  }
  __syncthreads();
  {
    const int r = threadIdx.x >> 2, part = threadIdx.x & 3;
    const double* xr = rows + r * pitch;
    double acc = 0.0;
    for (int d = part; d < D; d += 4) acc = fma(xr[d], xr[d], acc);
    const double p1 = __shfl_down_sync(0xFFFFFFFFu, acc, 1);
    const double p2 = __shfl_down_sync(0xFFFFFFFFu, acc, 2);
    const double p3 = __shfl_down_sync(0xFFFFFFFFu, acc, 3);
    if (part == 0) den[r] = fmaxf(round_dt(__fsqrt_rn(__double2float_rn(((acc + p1) + p2) + p3)), DT), eps);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kNormRows * CH; i += kNormThreads) {
    const int r = i / CH, c = i % CH;
    if (n0 + r >= N) continue;
    const double* xr = rows + r * pitch + c * epc;
    const float dn = den[r];
    float q[epc];
#pragma unroll
    for (int e = 0; e < epc; ++e) q[e] = round_dt(__fdiv_rn((float)xr[e], dn), DT);
    uint4 out;
    if constexpr (DT == LI_DTYPE_FP32) {
      out = make_uint4(__float_as_uint(q[0]), __float_as_uint(q[1]), __float_as_uint(q[2]), __float_as_uint(q[3]));
    } else {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t lo = DT == LI_DTYPE_BF16 ? (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(q[2 * e]))
                                                : (uint32_t)__half_as_ushort(__float2half_rn(q[2 * e]));
        const uint32_t hi = DT == LI_DTYPE_BF16 ? (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(q[2 * e + 1]))
                                                : (uint32_t)__half_as_ushort(__float2half_rn(q[2 * e + 1]));
        w[e] = lo | (hi << 16);
      }
      out = make_uint4(w[0], w[1], w[2], w[3]);
    }
    reinterpret_cast<uint4*>(y + (b * y_b + h * y_h + (int64_t)(n0 + r) * y_n) * es)[c] = out;
  }
}

template <int DT>
li_status launch_normalize(const li_view4* x, li_view4* y, int64_t B, int64_t H, int64_t N, int64_t D, float eps,
                           cudaStream_t stream) {
  const size_t smem = (size_t)kNormRows * (D + 1) * 8 + kNormRows * 4;
  static std::atomic<uint64_t> configured{0};
  if (li_status st = once_per_device(configured, [] {
        return cuda_status(cudaFuncSetAttribute(normalize_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                (int)(kNormRows * (kMaxD + 1) * 8 + kNormRows * 4)),
                           "normalize smem attribute");
      })) return st;
  normalize_kernel<DT><<<dim3((unsigned)ceil_div(N, kNormRows), (unsigned)(B * H)), kNormThreads, smem, stream>>>(
      static_cast<const uint8_t*>(x->data), x->stride[0], x->stride[1], x->stride[2], static_cast<uint8_t*>(y->data),
      y->stride[0], y->stride[1], y->stride[2], (int)H, (int)N, (int)D, eps);
  return launched("normalize_kernel launch");
}
}  // namespace
}  // namespace li

extern "C" li_status li_normalize_rows(const li_view4* x, li_view4* y, void* stream) {
  if (!x || !y) return fail(LI_ERR_INVALID_ARG, "x and y are required");
  const int64_t B = x->shape[0], H = x->shape[1], N = x->shape[2], D = x->shape[3];
  const int dt = x->dtype;
  if (li_status st = check_vec_view(x->data, x->stride, 4, dt, D, "x")) return st;
  if (li_status st = check_vec_view(y->data, y->stride, 4, y->dtype, D, "y")) return st;
  if (y->dtype != dt) return fail(LI_ERR_INVALID_ARG, "y dtype differs from x");
  for (int i = 0; i < 4; ++i)
    if (y->shape[i] != x->shape[i]) return fail(LI_ERR_SHAPE, "y shape differs from x");
  if (D > kMaxD) return fail(LI_ERR_UNSUPPORTED, "D=%lld", (long long)D);
  if (B * H == 0 || N == 0) return LI_OK;
  const float eps = dt == LI_DTYPE_FP32 ? 1e-12f
                  : dt == LI_DTYPE_BF16 ? __bfloat162float(__float2bfloat16_rn(1e-12f))
                                        : __half2float(__float2half_rn(1e-12f));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dt == LI_DTYPE_BF16) return launch_normalize<LI_DTYPE_BF16>(x, y, B, H, N, D, eps, st);
  if (dt == LI_DTYPE_FP16) return launch_normalize<LI_DTYPE_FP16>(x, y, B, H, N, D, eps, st);
  return launch_normalize<LI_DTYPE_FP32>(x, y, B, H, N, D, eps, st);
}

extern "C" li_status li_select_budget(const li_select_params* p, int64_t n_q_blocks, int64_t n_k_blocks,
                                      int32_t* n_text_blocks, int32_t* budget) {
  int32_t nprot;
  if (!n_text_blocks || !budget) return fail(LI_ERR_INVALID_ARG, "null output");
  return budget_of(p, n_q_blocks, n_k_blocks, n_text_blocks, budget, &nprot);
}

namespace li {
namespace {
// Validates the arguments of a selection and fills the kernel arguments.
li_status prepare_select(const li_view4* q_pool, const li_view4* k_pool, const li_select_params* p,
                         const li_view4* score_bias, li_index_view* out, li_view4* rank_out, SelArgs& a,
                         int64_t& B, int64_t& H) {
  if (!q_pool || !k_pool || !p) return fail(LI_ERR_INVALID_ARG, "q_pool, k_pool and params are required");
  B = q_pool->shape[0]; H = q_pool->shape[1];
  const int64_t Nq = q_pool->shape[2], D = q_pool->shape[3];
  const int64_t Nk = k_pool->shape[2];
  const int dt = q_pool->dtype;
  if (B < 0 || H < 0 || Nq < 0 || Nk < 0)
    return fail(LI_ERR_SHAPE, "pool shapes must be non-negative (B=%lld H=%lld Nq=%lld Nk=%lld)", (long long)B,
                (long long)H, (long long)Nq, (long long)Nk);
  if (!valid_dtype(dt) || k_pool->dtype != dt) return fail(LI_ERR_INVALID_ARG, "pool dtypes must match");
  if (k_pool->shape[0] != B || k_pool->shape[1] != H || k_pool->shape[3] != D)
    return fail(LI_ERR_SHAPE, "k_pool shape does not match q_pool");
  if (li_status st = check_vec_view(q_pool->data, q_pool->stride, 4, dt, D, "q_pool")) return st;
  if (li_status st = check_vec_view(k_pool->data, k_pool->stride, 4, dt, D, "k_pool")) return st;
  if (D <= 0 || D > kMaxD || D % 4) return fail(LI_ERR_UNSUPPORTED, "D=%lld", (long long)D);
  if (p->metric < LI_METRIC_COSINE || p->metric > LI_METRIC_DOT) return fail(LI_ERR_INVALID_ARG, "metric");
  int32_t ntxt, kb, nprot;
  if (li_status st = budget_of(p, Nq, Nk, &ntxt, &kb, &nprot)) return st;
  if (li_status st = check_index_out(out, B, H, Nq, (int64_t)ntxt + kb)) return st;
  if (p->mode == LI_SELECT_BIDIR) {
    if (p->grid_k[1] <= 0 || p->grid_k[2] <= 0) return fail(LI_ERR_INVALID_ARG, "grid_k");
    if (p->q_block_offset < 0 || p->q_block_offset + Nq > Nk)
      return fail(LI_ERR_SHAPE, "query rows [%d, %lld) fall outside the %lld key blocks", p->q_block_offset,
                  (long long)(p->q_block_offset + Nq), (long long)Nk);
  }
  if (Nk > (1 << 24)) return fail(LI_ERR_UNSUPPORTED, "too many key blocks");
  memset(&a, 0, sizeof(a));
  a.qp = static_cast<const uint8_t*>(q_pool->data);
  a.q_b = q_pool->stride[0]; a.q_h = q_pool->stride[1]; a.q_n = q_pool->stride[2];
  a.kp = static_cast<const uint8_t*>(k_pool->data);
  a.k_b = k_pool->stride[0]; a.k_h = k_pool->stride[1]; a.k_n = k_pool->stride[2];
  if (score_bias) {
    if (score_bias->dtype != LI_DTYPE_FP32) return fail(LI_ERR_INVALID_ARG, "score_bias must be fp32");
    if (score_bias->shape[0] != B || score_bias->shape[1] != H || score_bias->shape[2] != Nq ||
        score_bias->shape[3] != Nk)
      return fail(LI_ERR_SHAPE, "score_bias must be [B,H,Nq,Nk] (strides may be 0)");
    a.bias = static_cast<const float*>(score_bias->data);
    a.x_b = score_bias->stride[0]; a.x_h = score_bias->stride[1];
    a.x_q = score_bias->stride[2]; a.x_k = score_bias->stride[3];
  }
  a.idx = out->indices; a.i_b = out->stride[0]; a.i_h = out->stride[1]; a.i_q = out->stride[2]; a.i_s = out->stride[3];
  a.cnt = out->counts; a.c_b = out->count_stride[0]; a.c_h = out->count_stride[1]; a.c_q = out->count_stride[2];
  if (rank_out) {
    if (rank_out->dtype != LI_DTYPE_FP32) return fail(LI_ERR_INVALID_ARG, "rank_out must be fp32");
    if (rank_out->shape[0] != B || rank_out->shape[1] != H || rank_out->shape[2] != Nq || rank_out->shape[3] != Nk)
      return fail(LI_ERR_SHAPE, "rank_out must be [B,H,Nq,Nk]");
    a.rank = static_cast<float*>(rank_out->data);
    a.r_b = rank_out->stride[0]; a.r_h = rank_out->stride[1]; a.r_q = rank_out->stride[2]; a.r_k = rank_out->stride[3];
  }
  a.H = (int)H; a.D = (int)D; a.Nq = (int)Nq; a.Nk = (int)Nk; a.dtype = dt; a.metric = p->metric; a.mode = p->mode;
  a.n_prot = nprot; a.g_nh = p->grid_k[1]; a.g_nw = p->grid_k[2]; a.q_off = p->q_block_offset;
  a.k_budget = kb; a.ntxt = ntxt;
  int ib = 1;
  while ((1ll << ib) < Nk) ++ib;
  a.idx_bits = ib;
  a.key_bits = dt == LI_DTYPE_FP32 ? 32 : 16;
  a.scale = (float)(1.0 / std::sqrt((double)D));
  a.eps = dt == LI_DTYPE_FP32 ? 1e-12f
        : dt == LI_DTYPE_BF16 ? __bfloat162float(__float2bfloat16_rn(1e-12f))
                              : __half2float(__float2half_rn(1e-12f));
  if (p->mode == LI_SELECT_DECODE) {
    a.big = 1e6f;
  } else {
    const float one_e6 = 1.0f * 1e6f;
    a.big = dt == LI_DTYPE_FP32 ? one_e6
          : dt == LI_DTYPE_BF16 ? __bfloat162float(__float2bfloat16_rn(one_e6))
                                : __half2float(__float2half_rn(one_e6));
  }
  return LI_OK;
}

// SMs of the current device (148 on B200 when the query fails).
int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Key scratch of the two-kernel path: B*H*Nq*Nk 32-bit keys. Saturates at
// INT64_MAX instead of overflowing (no caller can hold that much).
int64_t select_ws_bytes(int64_t B, int64_t H, int64_t Nq, int64_t Nk) {
  int64_t n = 4;
  for (int64_t f : {B, H, Nq, Nk}) {
    if (f < 0 || __builtin_mul_overflow(n, f, &n)) return INT64_MAX;
  }
  return n;
}

// Shared memory of topk_kernel: the 256-bin histogram, scan scratch and the key row.
size_t topk_smem(int64_t Nk) { return (size_t)(256 + 16) * 4 + (size_t)4 * Nk; }

// Single-kernel selection (no workspace).
li_status launch_single(SelArgs& a, int64_t B, int64_t H, cudaStream_t s) {
  const int64_t D = a.D, Nk = a.Nk, Nq = a.Nq;
  auto smem_of = [&](int r) {
    return (size_t)8 * ((size_t)r * (D + 1) + (size_t)kChunkRows * (D + 1)) + (size_t)4 * r * Nk;
  };
  int R = 4;
  while (R > 1 && smem_of(R) > kSmemBudget) R >>= 1;
  if (smem_of(R) > kSmemBudget)
    return fail(LI_ERR_UNSUPPORTED, "%lld key blocks exceed the selection kernel's shared memory", (long long)Nk);
  if (Nq < R) R = Nq >= 4 ? 4 : (Nq >= 2 ? 2 : 1);
  a.R = R;
  const size_t smem = smem_of(R);
  dim3 grid((unsigned)ceil_div(Nq, R), (unsigned)(B * H));
  switch (R) {
    case 4: return launch_select<4>(a, grid, smem, s);
    case 2: return launch_select<2>(a, grid, smem, s);
    default: return launch_select<1>(a, grid, smem, s);
  }
}

// Two-kernel selection through `keys` (B*H*Nq*Nk uint32).
li_status launch_two(SelArgs& a, int64_t B, int64_t H, uint32_t* keys, cudaStream_t s) {
  static std::atomic<uint64_t> configured{0};
  if (li_status st = once_per_device(configured, [] {
        if (li_status e = cuda_status(cudaFuncSetAttribute(score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                           (int)((kScoreRows + kScoreKeys) * (kMaxD + 1) * 8)),
                                      "score_kernel smem attribute")) return e;
        return cuda_status(cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                (int)kSmemBudget), "topk_kernel smem attribute");
      })) return st;
  if (a.metric == LI_METRIC_COSINE || a.D % kTileD) {
    // In-kernel normalisation needs whole rows staged.
    const size_t smem1 = (size_t)(kScoreRows + kScoreKeys) * (a.D + 1) * 8;
    score_kernel<<<dim3((unsigned)ceil_div(a.Nq, kScoreRows), (unsigned)ceil_div(a.Nk, kScoreKeys), (unsigned)(B * H)),
                   128, smem1, s>>>(a, keys);
    if (li_status st = launched("score_kernel launch")) return st;
  } else {
    // 128-key tiles unless they leave the grid under two waves of the GPU.
    const int64_t ctas128 = ceil_div(a.Nq, kTileRows) * ceil_div(a.Nk, kTileKeysMax) * B * H;
    const int M = ctas128 < 2 * (int64_t)sm_count() ? 1 : 2;
    const int tile_keys = 64 * M;
    const size_t smem1 = ((size_t)kTileRows * (kTileD + 2) + (size_t)tile_keys * (kTileD + 1)) * 8;
    const dim3 grid((unsigned)ceil_div(a.Nq, kTileRows), (unsigned)ceil_div(a.Nk, tile_keys), (unsigned)(B * H));
    if (M == 1) {
      if (a.dtype == LI_DTYPE_BF16) score_tile_kernel<LI_DTYPE_BF16, 1><<<grid, kTileThreads, smem1, s>>>(a, keys);
      else if (a.dtype == LI_DTYPE_FP16) score_tile_kernel<LI_DTYPE_FP16, 1><<<grid, kTileThreads, smem1, s>>>(a, keys);
      else score_tile_kernel<LI_DTYPE_FP32, 1><<<grid, kTileThreads, smem1, s>>>(a, keys);
    } else {
      if (a.dtype == LI_DTYPE_BF16) score_tile_kernel<LI_DTYPE_BF16, 2><<<grid, kTileThreads, smem1, s>>>(a, keys);
      else if (a.dtype == LI_DTYPE_FP16) score_tile_kernel<LI_DTYPE_FP16, 2><<<grid, kTileThreads, smem1, s>>>(a, keys);
      else score_tile_kernel<LI_DTYPE_FP32, 2><<<grid, kTileThreads, smem1, s>>>(a, keys);
    }
    if (li_status st = launched("score_tile_kernel launch")) return st;
  }
  const size_t smem2 = topk_smem(a.Nk);
  topk_kernel<<<dim3((unsigned)a.Nq, (unsigned)(B * H)), kTopkThreads, smem2, s>>>(a, keys);
  return launched("topk_kernel launch");
}
}  // namespace
}  // namespace li

extern "C" li_status li_select_workspace_bytes(int64_t batch, int64_t heads, int64_t n_q_blocks, int64_t n_k_blocks,
                                               int64_t* bytes) {
  if (!bytes) return fail(LI_ERR_INVALID_ARG, "bytes is required");
  if (batch < 0 || heads < 0 || n_q_blocks < 0 || n_k_blocks < 0) return fail(LI_ERR_SHAPE, "negative shape");
  *bytes = topk_smem(n_k_blocks) <= kSmemBudget ? select_ws_bytes(batch, heads, n_q_blocks, n_k_blocks) : 0;
  return LI_OK;
}

extern "C" li_status li_select_blocks(const li_view4* q_pool, const li_view4* k_pool,
                                      const li_select_params* p, const li_view4* score_bias,
                                      li_index_view* out, li_view4* rank_out, void* workspace,
                                      int64_t workspace_bytes, void* stream) {
  SelArgs a;
  int64_t B, H;
  if (li_status st = prepare_select(q_pool, k_pool, p, score_bias, out, rank_out, a, B, H)) return st;
  if (B * H == 0 || a.Nq == 0) return LI_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t need = select_ws_bytes(B, H, a.Nq, a.Nk);
  if (workspace && workspace_bytes >= need && topk_smem(a.Nk) <= kSmemBudget && aligned16(workspace))
    return launch_two(a, B, H, static_cast<uint32_t*>(workspace), s);
  return launch_single(a, B, H, s);
}

// ---------------------------------------------------------------------------
// Two-kernel selection through a scratch buffer the library owns.
//
// Some callers have no device allocator to hand a workspace from: a host
// binding over the C ABI (cgo, JNI, ctypes) that links no torch, or a serving
// loop that must not call cudaMalloc mid-step because it synchronises the
// device and stalls every other stream. For them the sort keys of the
// two-kernel path live in a fixed array in this module's global memory, which
// is reserved when the module loads, so the call itself allocates nothing.
// ---------------------------------------------------------------------------
static_assert(LI_SELECT_STATIC_SCRATCH_BYTES % 4 == 0, "scratch holds 32-bit keys");
// One 32-bit key per (b, h, query row, key block). The score kernel writes
// every word the top-k kernel reads within the same call, so no part of it has
// to start at zero and nothing carries over between calls.
static __device__ __align__(256) uint32_t g_select_scratch[LI_SELECT_STATIC_SCRATCH_BYTES / 4];

namespace li {
namespace {
constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mu;
uint32_t* g_scratch_addr[kMaxScratchDevices];

// Device address of g_select_scratch on the current device, looked up once per
// device. The first lookup may load this module onto the device.
li_status static_scratch(uint32_t** addr) {
  int dev = 0;
  if (li_status st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice")) return st;
  if (dev < 0 || dev >= kMaxScratchDevices) return fail(LI_ERR_UNSUPPORTED, "device ordinal %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (li_status st = cuda_status(cudaGetSymbolAddress(&p, g_select_scratch),
                                   "cudaGetSymbolAddress(selection scratch)")) return st;
    if (!p || !aligned16(p)) return fail(LI_ERR_CUDA, "selection scratch address is not 16-byte aligned");
    g_scratch_addr[dev] = static_cast<uint32_t*>(p);
  }
  *addr = g_scratch_addr[dev];
  return LI_OK;
}
}  // namespace
}  // namespace li

extern "C" li_status li_select_blocks_static(const li_view4* q_pool, const li_view4* k_pool,
                                             const li_select_params* p, const li_view4* score_bias,
                                             li_index_view* out, li_view4* rank_out, void* stream) {
  SelArgs a;
  int64_t B, H;
  if (li_status st = prepare_select(q_pool, k_pool, p, score_bias, out, rank_out, a, B, H)) return st;
  const int64_t need = select_ws_bytes(B, H, a.Nq, a.Nk);
  if (need > LI_SELECT_STATIC_SCRATCH_BYTES)
    return fail(LI_ERR_UNSUPPORTED,
                "selection of %lld x %lld x %lld x %lld (batch x heads x query blocks x key blocks) needs %lld "
                "bytes of scratch; the static buffer holds %lld (use li_select_blocks with a workspace)",
                (long long)B, (long long)H, (long long)a.Nq, (long long)a.Nk, (long long)need,
                (long long)LI_SELECT_STATIC_SCRATCH_BYTES);
  if (topk_smem(a.Nk) > kSmemBudget)
    return fail(LI_ERR_UNSUPPORTED, "%lld key blocks exceed the top-k kernel's shared memory", (long long)a.Nk);
  uint32_t* scratch = nullptr;
  if (li_status st = static_scratch(&scratch)) return st;
  if (B * H == 0 || a.Nq == 0) return LI_OK;
  return launch_two(a, B, H, scratch, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// Ranking alone on given scores.
// ---------------------------------------------------------------------------
namespace li {
namespace {
struct RankArgs {
  const float* sc; int64_t s_b, s_h, s_q, s_k;
  int32_t* idx; int64_t i_b, i_h, i_q, i_s;
  int32_t* cnt; int64_t c_b, c_h, c_q;
  int32_t H, Nq, Nk, dtype, k, ntxt, idx_bits, key_bits;
};

__global__ void __launch_bounds__(kThreads) rank_kernel(const RankArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int qi = blockIdx.x * kWarps + warp;
  const int b = blockIdx.y / a.H, h = blockIdx.y % a.H;
  if (qi >= a.Nq) return;
  uint32_t* rk = keys + warp * a.Nk;
  const float* row = a.sc + b * a.s_b + h * a.s_h + (int64_t)qi * a.s_q;
  for (int j = lane; j < a.Nk; j += 32) rk[j] = radix_key(row[(int64_t)j * a.s_k], a.dtype);
  __syncwarp();
  const uint64_t low_mask = (1ull << a.idx_bits) - 1ull;
  uint64_t thr = 0;
  if (a.k > 0 && a.k < a.Nk) {
    for (int bit = a.key_bits + a.idx_bits - 1; bit >= 0; --bit) {
      const uint64_t cand = thr | (1ull << bit);
      int c = 0;
      for (int j = lane; j < a.Nk; j += 32) c += (((uint64_t)rk[j] << a.idx_bits) | (low_mask - (uint64_t)j)) >= cand;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
      if (c >= a.k) thr = cand;
    }
  }
  int32_t* out = a.idx + b * a.i_b + h * a.i_h + (int64_t)qi * a.i_q;
  for (int t = lane; t < a.ntxt; t += 32) out[(int64_t)t * a.i_s] = t;
  int pos = 0;
  if (a.k > 0) {
    for (int base = 0; base < a.Nk; base += 32) {
      const int j = base + lane;
      bool sel = false;
      if (j < a.Nk) sel = (a.k >= a.Nk) || ((((uint64_t)rk[j] << a.idx_bits) | (low_mask - (uint64_t)j)) >= thr);
      const unsigned m = __ballot_sync(0xFFFFFFFFu, sel);
      if (sel) out[(int64_t)(a.ntxt + pos + __popc(m & ((1u << lane) - 1u))) * a.i_s] = j + a.ntxt;
      pos += __popc(m);
    }
  }
  if (lane == 0) a.cnt[b * a.c_b + h * a.c_h + (int64_t)qi * a.c_q] = a.ntxt + a.k;
}
}  // namespace
}  // namespace li

extern "C" li_status li_rank_blocks(const li_view4* rank_scores, int32_t score_dtype, int32_t k,
                                    int32_t text_len, int32_t bs, li_index_view* out, void* stream) {
  if (!rank_scores) return fail(LI_ERR_INVALID_ARG, "rank_scores required");
  if (rank_scores->dtype != LI_DTYPE_FP32) return fail(LI_ERR_INVALID_ARG, "rank_scores must be fp32 storage");
  if (!valid_dtype(score_dtype)) return fail(LI_ERR_INVALID_ARG, "score_dtype");
  if (bs <= 0 || text_len < 0) return fail(LI_ERR_INVALID_ARG, "bs / text_len");
  const int64_t B = rank_scores->shape[0], H = rank_scores->shape[1], Nq = rank_scores->shape[2],
                Nk = rank_scores->shape[3];
  if (k < 0 || k > Nk) return fail(LI_ERR_OUT_OF_BOUNDS, "k=%d outside [0, %lld]", k, (long long)Nk);
  const int32_t ntxt = (int32_t)((text_len + bs - 1) / bs);
  if (li_status st = check_index_out(out, B, H, Nq, (int64_t)ntxt + k)) return st;
  const size_t smem = (size_t)kWarps * Nk * 4;
  if (smem > kSmemBudget) return fail(LI_ERR_UNSUPPORTED, "too many key blocks for li_rank_blocks");
  if (B * H == 0 || Nq == 0) return LI_OK;
  RankArgs a;
  memset(&a, 0, sizeof(a));
  a.sc = static_cast<const float*>(rank_scores->data);
  a.s_b = rank_scores->stride[0]; a.s_h = rank_scores->stride[1]; a.s_q = rank_scores->stride[2]; a.s_k = rank_scores->stride[3];
  a.idx = out->indices; a.i_b = out->stride[0]; a.i_h = out->stride[1]; a.i_q = out->stride[2]; a.i_s = out->stride[3];
  a.cnt = out->counts; a.c_b = out->count_stride[0]; a.c_h = out->count_stride[1]; a.c_q = out->count_stride[2];
  a.H = (int)H; a.Nq = (int)Nq; a.Nk = (int)Nk; a.dtype = score_dtype; a.k = k; a.ntxt = ntxt;
  int ib = 1;
  while ((1ll << ib) < Nk) ++ib;
  a.idx_bits = ib;
  a.key_bits = score_dtype == LI_DTYPE_FP32 ? 32 : 16;
  static std::atomic<uint64_t> configured{0};
  if (li_status st = once_per_device(configured, [] {
        return cuda_status(cudaFuncSetAttribute(rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                (int)kSmemBudget), "rank_kernel smem attribute");
      })) return st;
  rank_kernel<<<dim3((unsigned)ceil_div(Nq, kWarps), (unsigned)(B * H)), kThreads, smem,
                static_cast<cudaStream_t>(stream)>>>(a);
  return launched("rank_kernel launch");
}
