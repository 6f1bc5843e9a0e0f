// Block selection: pooled-score GEMM, protection bias, top-k, sorted emit.
//
// One CTA (8 warps) handles R <= 8 query rows of one (b, h). The query rows
// and then the key rows, 32 at a time, are staged in shared memory as floats
// with coalesced 16-byte loads ('cosine' normalises them there). Warp r forms
// the dot products of query row r with the 32 staged key rows, one per lane.
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

#include "li_common.cuh"

namespace li {
namespace {

constexpr int kThreads = 256;
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
__device__ __forceinline__ double dot4(const float* x, const float* y, int D) {
  double p0 = 0.0, p1 = 0.0, p2 = 0.0, p3 = 0.0;
  for (int d = 0; d < D; d += 4) {
    p0 = fma((double)x[d], (double)y[d], p0);
    p1 = fma((double)x[d + 1], (double)y[d + 1], p1);
    p2 = fma((double)x[d + 2], (double)y[d + 2], p2);
    p3 = fma((double)x[d + 3], (double)y[d + 3], p3);
  }
  return ((p0 + p1) + p2) + p3;
}

// 16-byte chunk of a pooled row -> floats (exact widening).
__device__ __forceinline__ void widen_chunk(const uint4& v, int dt, float* dst) {
  const int epc = dt == LI_DTYPE_FP32 ? 4 : 8;
  for (int e = 0; e < epc; ++e) dst[e] = chunk_elem(v, e, dt);
}

constexpr int kChunkRows = 32;

template <int R>
__global__ void __launch_bounds__(kThreads) select_kernel(const SelArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int pitch = a.D + 1;                                   // bank-conflict-free row pitch
  float* qs = reinterpret_cast<float*>(smem);                   // [R][pitch]
  float* ks = qs + R * pitch;                                   // [kChunkRows][pitch]
  float* kden = ks + kChunkRows * pitch;                        // [kChunkRows]
  float* qden = kden + kChunkRows;                              // [R]
  uint32_t* keys = reinterpret_cast<uint32_t*>(qden + R);       // [R][Nk]
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
  if (cosine) {
    if (tid < R) {
      const float* x = qs + tid * pitch;
      qden[tid] = fmaxf(round_dt(__fsqrt_rn(__double2float_rn(dot4(x, x, a.D))), a.dtype), a.eps);
    }
    __syncthreads();
    for (int i = tid; i < R * a.D; i += kThreads) {
      const int r = i / a.D, d = i % a.D;
      qs[r * pitch + d] = round_dt(__fdiv_rn(qs[r * pitch + d], qden[r]), a.dtype);
    }
  }

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
      if (tid < kChunkRows) {
        const float* x = ks + tid * pitch;
        kden[tid] = fmaxf(round_dt(__fsqrt_rn(__double2float_rn(dot4(x, x, a.D))), a.dtype), a.eps);
      }
      __syncthreads();
      for (int i = tid; i < kChunkRows * a.D; i += kThreads) {
        const int r = i / a.D, d = i % a.D;
        ks[r * pitch + d] = round_dt(__fdiv_rn(ks[r * pitch + d], kden[r]), a.dtype);
      }
      __syncthreads();
    }
    // Warp r forms the dot products of query row r with the 32 staged key rows.
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
cudaError_t launch_select(const SelArgs& a, dim3 grid, size_t smem, cudaStream_t s) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(select_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kSmemBudget);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  select_kernel<R><<<grid, kThreads, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace
}  // namespace li

using namespace li;

extern "C" li_status li_select_budget(const li_select_params* p, int64_t n_q_blocks, int64_t n_k_blocks,
                                      int32_t* n_text_blocks, int32_t* budget) {
  int32_t nprot;
  if (!n_text_blocks || !budget) return fail(LI_ERR_INVALID_ARG, "null output");
  return budget_of(p, n_q_blocks, n_k_blocks, n_text_blocks, budget, &nprot);
}

extern "C" li_status li_select_blocks(const li_view4* q_pool, const li_view4* k_pool,
                                      const li_select_params* p, const li_view4* score_bias,
                                      li_index_view* out, li_view4* rank_out, void* stream) {
  if (!q_pool || !k_pool || !p) return fail(LI_ERR_INVALID_ARG, "q_pool, k_pool and params are required");
  const int64_t B = q_pool->shape[0], H = q_pool->shape[1], Nq = q_pool->shape[2], D = q_pool->shape[3];
  const int64_t Nk = k_pool->shape[2];
  const int dt = q_pool->dtype;
  if (!valid_dtype(dt) || k_pool->dtype != dt) return fail(LI_ERR_INVALID_ARG, "pool dtypes must match");
  if (k_pool->shape[0] != B || k_pool->shape[1] != H || k_pool->shape[3] != D)
    return fail(LI_ERR_SHAPE, "k_pool shape does not match q_pool");
  if (li_status st = check_vec_view(q_pool->data, q_pool->stride, 4, dt, D, "q_pool")) return st;
  if (li_status st = check_vec_view(k_pool->data, k_pool->stride, 4, dt, D, "k_pool")) return st;
  if (D <= 0 || D > kMaxD) return fail(LI_ERR_UNSUPPORTED, "D=%lld", (long long)D);
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
  if (B * H == 0 || Nq == 0) return LI_OK;
  SelArgs a;
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
  // Rows per CTA: as many (<= 8) as fit the shared-memory budget.
  auto smem_of = [&](int r) {
    return (size_t)4 * ((size_t)r * (D + 1) + (size_t)kChunkRows * (D + 1) + kChunkRows + r + (size_t)r * Nk);
  };
  int R = 8;
  while (R > 1 && smem_of(R) > kSmemBudget) R >>= 1;
  if (smem_of(R) > kSmemBudget)
    return fail(LI_ERR_UNSUPPORTED, "%lld key blocks exceed the selection kernel's shared memory", (long long)Nk);
  if (Nq < R) R = Nq >= 4 ? 4 : (Nq >= 2 ? 2 : 1);
  a.R = R;
  const size_t smem = smem_of(R);
  dim3 grid((unsigned)ceil_div(Nq, R), (unsigned)(B * H));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (R) {
    case 8: e = launch_select<8>(a, grid, smem, s); break;
    case 4: e = launch_select<4>(a, grid, smem, s); break;
    case 2: e = launch_select<2>(a, grid, smem, s); break;
    default: e = launch_select<1>(a, grid, smem, s); break;
  }
  return cuda_status(e, "select_kernel launch");
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
  static bool configured = false;
  if (!configured) {
    if (li_status st = cuda_status(cudaFuncSetAttribute(rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                        (int)kSmemBudget), "rank_kernel smem attribute")) return st;
    configured = true;
  }
  rank_kernel<<<dim3((unsigned)ceil_div(Nq, kWarps), (unsigned)(B * H)), kThreads, smem,
                static_cast<cudaStream_t>(stream)>>>(a);
  return cuda_status(cudaGetLastError(), "rank_kernel launch");
}
