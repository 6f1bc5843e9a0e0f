// HBM-bound layout kernels: 3D tiling + block mean pooling (with the fused
// memory-pruning frame gather), text blocks, untiling, and the stand-alone
// retained-frame gather.
//
// All four move 16-byte chunks: a row of D elements is CH = D*elem/16 chunks.
// A CTA of 8*CH threads (per stream) covers one 3D block: thread (g, c) copies
// chunk c of rows g, g+8, g+16, ... and, for the pooled stream, accumulates
// those rows in fp64. The eight row-group partial sums are then combined in
// order g = 0..7 — the summation order the CPU oracle restates.
#include <algorithm>
#include <cstring>

#include "li_common.cuh"

namespace li {
namespace {

constexpr int kMaxD = 256;
constexpr int kUnroll = 8;       // 16-byte copies in flight per thread (gather)
constexpr int kPoolUnroll = 4;   // rows in flight per thread (pool / tile); 4 keeps 8 CTAs of 128 threads resident

struct TileArgs {
  const uint8_t* src[2];
  int64_t s_b[2], s_h[2], s_l[2];
  uint8_t* dst[2];
  int64_t d_b[2], d_h[2], d_n[2], d_r[2];
  uint8_t* pool;
  int64_t p_b, p_h, p_n;
  const int32_t* frame_ids;
  uint32_t* err;
  int64_t dst_off, pool_off;
  int32_t src_frames;
  int32_t nstreams;
  int32_t flat;        // 1: flat token rows (text blocks), 0: raster 3D blocks
  int32_t n_tokens;    // flat: valid tokens
  int32_t T, LH, LW, tt, th, tw, nh, nw;
  int32_t H, bs, D, dtype, CH;
  int32_t normalize;   // 1: store F.normalize of the block mean instead of the mean
  float eps;           // dtype(1e-12), the clamp of the normalisation
};

// Raster token of row r of block `blk` (-1: padding or a rejected frame id).
__device__ __forceinline__ int64_t token_of(const TileArgs& a, int blk, int r, bool& bad_frame) {
  bad_frame = false;
  if (a.flat) {
    const int64_t tok = (int64_t)blk * a.bs + r;
    return tok < a.n_tokens ? tok : -1;
  }
  const int cw = blk % a.nw;
  const int rem = blk / a.nw;
  const int ch = rem % a.nh;
  const int ct = rem / a.nh;
  const int ow = r % a.tw;
  const int rr = r / a.tw;
  const int oh = rr % a.th;
  const int ot = rr / a.th;
  const int t = ct * a.tt + ot, h = ch * a.th + oh, w = cw * a.tw + ow;
  if (t >= a.T || h >= a.LH || w >= a.LW) return -1;
  int64_t f = t;
  if (a.frame_ids) {
    f = a.frame_ids[t];
    if (f < 0 || f >= a.src_frames) {
      bad_frame = true;
      return -1;
    }
  }
  return (f * a.LH + h) * (int64_t)a.LW + w;
}

constexpr int kMaxBS = 1024;  // tokens per 3D block (the pooling CTA's row table)

// DT is the element type (LI_DTYPE_*), fixed at compile time so the per-element
// widening carries no dtype branches.
template <int DT>
__device__ __forceinline__ void tile_pool_block(const TileArgs& a, const int blk, const int bh, uint8_t* smem) {
  double* partial = reinterpret_cast<double*>(smem);                // [8][D]
  int32_t* rowtok = reinterpret_cast<int32_t*>(partial + 8 * a.D);  // token of each row, -1 = zero row
  float* prow = reinterpret_cast<float*>(rowtok + a.bs);            // [D] dtype-rounded means
  double* nrm = reinterpret_cast<double*>(smem);                    // [4] partial sums (reuses partial)
  const int b = bh / a.H, h = bh % a.H;
  const int per_stream = 8 * a.CH;
  const int s = threadIdx.x / per_stream;
  const int t2 = threadIdx.x % per_stream;
  const int g = t2 / a.CH, c = t2 % a.CH;
  constexpr int es = DT == LI_DTYPE_FP32 ? 4 : 2;
  constexpr int epc = 16 / es;
  const bool pooling = (s == 0) && (a.pool != nullptr);

  bool any_bad = false;
  for (int r = threadIdx.x; r < a.bs; r += blockDim.x) {
    bool bad;
    rowtok[r] = (int32_t)token_of(a, blk, r, bad);
    any_bad |= bad;
  }
  if (any_bad && a.err) atomicOr(a.err, (unsigned)LI_DEVERR_BAD_INDEX);
  __syncthreads();

  const uint8_t* src = a.src[s] + (b * a.s_b[s] + h * a.s_h[s]) * es + c * 16;
  const int64_t sl = a.s_l[s] * es;
  uint8_t* dst = a.dst[s] ? a.dst[s] + (b * a.d_b[s] + h * a.d_h[s] + (blk + a.dst_off) * a.d_n[s]) * es + c * 16
                          : nullptr;
  double acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.0;

  const int rows_per_thread = a.bs / 8;
  for (int i0 = 0; i0 < rows_per_thread; i0 += kPoolUnroll) {
    uint4 v[kPoolUnroll];
#pragma unroll
    for (int u = 0; u < kPoolUnroll; ++u) {
      v[u] = make_uint4(0, 0, 0, 0);
      const int i = i0 + u;
      if (i < rows_per_thread) {
        const int32_t tok = rowtok[g + 8 * i];
        if (tok >= 0) v[u] = __ldg(reinterpret_cast<const uint4*>(src + (int64_t)tok * sl));
      }
    }
#pragma unroll
    for (int u = 0; u < kPoolUnroll; ++u) {
      const int i = i0 + u;
      if (i < rows_per_thread) {
        if (dst) *reinterpret_cast<uint4*>(dst + (int64_t)(g + 8 * i) * a.d_r[s] * es) = v[u];
        if (pooling) {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (e < epc) acc[e] += (double)chunk_elem(v[u], e, DT);
        }
      }
    }
  }
  if (a.pool == nullptr) return;
  if (pooling) {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (e < epc) partial[g * a.D + c * epc + e] = acc[e];
  }
  __syncthreads();
  if (pooling && g == 0) {
    for (int e = 0; e < epc; ++e) {
      const int col = c * epc + e;
      double tot = partial[col];
#pragma unroll
      for (int gg = 1; gg < 8; ++gg) tot = tot + partial[gg * a.D + col];
      prow[col] = round_dt(__fdiv_rn(__double2float_rn(tot), (float)a.bs), DT);
    }
  }
  __syncthreads();
  uint8_t* pp = a.pool + (b * a.p_b + h * a.p_h + (blk + a.pool_off) * a.p_n) * es;
  if (!a.normalize) {
    if (pooling && g == 0)
      for (int e = 0; e < epc; ++e) store_dt(pp, c * epc + e, prow[c * epc + e], DT);
    return;
  }
  // F.normalize of the mean row: four interleaved fp64 partial sums of squares
  // (d mod 4, ascending d) combined in order, the selection's rounding chain.
  if (threadIdx.x < 4) {
    double acc = 0.0;
    for (int d = threadIdx.x; d < a.D; d += 4) acc = fma((double)prow[d], (double)prow[d], acc);
    nrm[threadIdx.x] = acc;
  }
  __syncthreads();
  if (pooling && g == 0) {
    const double sum = ((nrm[0] + nrm[1]) + nrm[2]) + nrm[3];
    const float den = fmaxf(round_dt(__fsqrt_rn(__double2float_rn(sum)), DT), a.eps);
    for (int e = 0; e < epc; ++e)
      store_dt(pp, c * epc + e, round_dt(__fdiv_rn(prow[c * epc + e], den), DT), DT);
  }
}

template <int DT>
__global__ void __launch_bounds__(512) tile_pool_kernel(const TileArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  tile_pool_block<DT>(a, blockIdx.x, blockIdx.y, smem);
}

// Several pooling jobs in one launch (e.g. a layer's q and the changed rows of
// its key pool): CTA i belongs to the job j with start[j] <= i < start[j+1] and
// pools block (i - start[j]) % nblk_j of (b, h) = (i - start[j]) / nblk_j.
constexpr int kMaxPoolJobs = 4;
struct TileMulti {
  TileArgs job[kMaxPoolJobs];
  int64_t start[kMaxPoolJobs + 1];
  int64_t nblk[kMaxPoolJobs];
  int32_t n;
};

template <int DT>
__global__ void __launch_bounds__(512) tile_pool_multi_kernel(const __grid_constant__ TileMulti m) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int64_t i = blockIdx.x;
  int j = 0;
  while (j + 1 < m.n && i >= m.start[j + 1]) ++j;
  const int64_t r = i - m.start[j];
  tile_pool_block<DT>(m.job[j], (int)(r % m.nblk[j]), (int)(r / m.nblk[j]), smem);
}

struct UntileArgs {
  const uint8_t* src;
  int64_t s_b, s_h, s_n, s_r;
  uint8_t* dst;
  int64_t d_b, d_h, d_l;
  int32_t T, LH, LW, tt, th, tw, nh, nw;
  int32_t H, bs, dtype, CH;
};

__global__ void untile_kernel(const UntileArgs a) {
  const int blk = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / a.H, h = bh % a.H;
  const int g = threadIdx.x / a.CH, c = threadIdx.x % a.CH;
  const int es = a.dtype == LI_DTYPE_FP32 ? 4 : 2;
  const uint8_t* src = a.src + (b * a.s_b + h * a.s_h + blk * a.s_n) * es + c * 16;
  uint8_t* dst = a.dst + (b * a.d_b + h * a.d_h) * es + c * 16;
  const int cw = blk % a.nw, rem = blk / a.nw, chh = rem % a.nh, ct = rem / a.nh;
  for (int r = g; r < a.bs; r += 8) {
    const int ow = r % a.tw, rr = r / a.tw, oh = rr % a.th, ot = rr / a.th;
    const int t = ct * a.tt + ot, hh = chh * a.th + oh, w = cw * a.tw + ow;
    if (t < a.T && hh < a.LH && w < a.LW) {
      const int64_t tok = ((int64_t)t * a.LH + hh) * a.LW + w;
      *reinterpret_cast<uint4*>(dst + tok * a.d_l * es) =
          __ldg(reinterpret_cast<const uint4*>(src + (int64_t)r * a.s_r * es));
    }
  }
}

struct GatherArgs {
  const uint8_t* src;
  int64_t s_b, s_h, s_l;
  uint8_t* dst;
  int64_t d_b, d_h, d_l;
  const int32_t* frame_ids;
  uint32_t* err;
  int32_t src_frames, frame_tokens, H, dtype, CH;
};

// One CTA per (kGatherRows-token piece of a retained frame, b*h): the frame's
// rows are split so that even a few heads and frames fill the GPU.
constexpr int kGatherRows = 64;
__global__ void __launch_bounds__(256) gather_frames_kernel(const GatherArgs a) {
  const int pieces = (a.frame_tokens + kGatherRows - 1) / kGatherRows;
  const int f = blockIdx.x / pieces, piece = blockIdx.x % pieces;
  const int bh = blockIdx.y;
  const int b = bh / a.H, h = bh % a.H;
  const int es = a.dtype == LI_DTYPE_FP32 ? 4 : 2;
  const int sf = a.frame_ids[f];
  const bool ok = sf >= 0 && sf < a.src_frames;
  if (!ok && threadIdx.x == 0 && a.err) atomicOr(a.err, (unsigned)LI_DEVERR_BAD_INDEX);
  const int r0 = piece * kGatherRows;
  const int nrows = min(kGatherRows, a.frame_tokens - r0);
  const uint8_t* src = a.src + (b * a.s_b + h * a.s_h + ((int64_t)sf * a.frame_tokens + r0) * a.s_l) * es;
  uint8_t* dst = a.dst + (b * a.d_b + h * a.d_h + ((int64_t)f * a.frame_tokens + r0) * a.d_l) * es;
  const int total = nrows * a.CH;
  for (int base = threadIdx.x; base < total; base += blockDim.x * kUnroll) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = base + u * blockDim.x;
      v[u] = make_uint4(0, 0, 0, 0);
      if (ok && i < total)
        v[u] = __ldg(reinterpret_cast<const uint4*>(src + ((int64_t)(i / a.CH) * a.s_l) * es + (i % a.CH) * 16));
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = base + u * blockDim.x;
      if (i < total)
        *reinterpret_cast<uint4*>(dst + ((int64_t)(i / a.CH) * a.d_l) * es + (i % a.CH) * 16) = v[u];
    }
  }
}

li_status check_grid(const li_grid3d& g) {
  if (g.T <= 0 || g.LH <= 0 || g.LW <= 0 || g.tt <= 0 || g.th <= 0 || g.tw <= 0)
    return fail(LI_ERR_SHAPE, "grid dims must be positive (T=%d LH=%d LW=%d tile=%d,%d,%d)", g.T, g.LH,
                g.LW, g.tt, g.th, g.tw);
  const int bs = g.tt * g.th * g.tw;
  if (bs % 8 || bs > kMaxBS)
    return fail(LI_ERR_UNSUPPORTED, "block size %d must be a multiple of 8 and <= %d", bs, kMaxBS);
  return LI_OK;
}

li_status fill_dst(TileArgs& a, int s, li_view5* d, int64_t B, int64_t H, int64_t D, int dtype,
                   int64_t nblk_needed, const char* name) {
  if (!d) { a.dst[s] = nullptr; return LI_OK; }
  li_status st = check_vec_view(d->data, d->stride, 5, d->dtype, D, name);
  if (st) return st;
  if (d->dtype != dtype) return fail(LI_ERR_INVALID_ARG, "%s: dtype differs from the source", name);
  if (d->shape[0] != B || d->shape[1] != H || d->shape[3] != a.bs || d->shape[4] != D)
    return fail(LI_ERR_SHAPE, "%s: expected [B=%lld,H=%lld,*,bs=%d,D=%lld]", name, (long long)B,
                (long long)H, a.bs, (long long)D);
  if (d->shape[2] < nblk_needed)
    return fail(LI_ERR_OUT_OF_BOUNDS, "%s: %lld blocks, need %lld", name, (long long)d->shape[2],
                (long long)nblk_needed);
  a.dst[s] = static_cast<uint8_t*>(d->data);
  a.d_b[s] = d->stride[0]; a.d_h[s] = d->stride[1]; a.d_n[s] = d->stride[2]; a.d_r[s] = d->stride[3];
  return LI_OK;
}

li_status launch_tile(TileArgs& a, int64_t nblk, int64_t B, int64_t H, void* stream) {
  if (nblk == 0 || B * H == 0) return LI_OK;
  if (nblk > 2147483647 || B * H > 65535) return fail(LI_ERR_SHAPE, "grid too large");
  dim3 grid((unsigned)nblk, (unsigned)(B * H));
  dim3 block(8 * a.CH * a.nstreams);
  const size_t smem = (size_t)8 * a.D * 8 + (size_t)a.bs * 4 + (size_t)a.D * 4;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a.dtype == LI_DTYPE_BF16) tile_pool_kernel<LI_DTYPE_BF16><<<grid, block, smem, st>>>(a);
  else if (a.dtype == LI_DTYPE_FP16) tile_pool_kernel<LI_DTYPE_FP16><<<grid, block, smem, st>>>(a);
  else tile_pool_kernel<LI_DTYPE_FP32><<<grid, block, smem, st>>>(a);
  return launched("tile_pool_kernel launch");
}

}  // namespace
}  // namespace li

using namespace li;

namespace li {
namespace {
// Validates one tiling / pooling job and fills its kernel arguments; `nblk`,
// `B`, `H` receive its grid. `*empty` is set when there is nothing to launch.
li_status prepare_tile(const li_view4* src0, const li_view4* src1, const int32_t* frame_ids, li_grid3d grid,
                       li_view5* dst0, li_view5* dst1, int64_t dst_block_offset, li_view4* pool,
                       int64_t pool_block_offset, int normalize, TileArgs& a, int64_t& nblk, int64_t& B_out,
                       int64_t& H_out, bool* empty) {
  *empty = false;
  if (!src0) return fail(LI_ERR_INVALID_ARG, "src0 is required");
  if ((src1 == nullptr) != (dst1 == nullptr)) return fail(LI_ERR_INVALID_ARG, "dst1 must be given iff src1 is");
  if (li_status st = check_grid(grid)) return st;
  const int64_t B = src0->shape[0], H = src0->shape[1], L = src0->shape[2], D = src0->shape[3];
  const int dtype = src0->dtype;
  if (li_status st = check_vec_view(src0->data, src0->stride, 4, dtype, D, "src0")) return st;
  if (D > kMaxD) return fail(LI_ERR_UNSUPPORTED, "D=%lld exceeds %d", (long long)D, kMaxD);
  const int64_t HW = (int64_t)grid.LH * grid.LW;
  if (L % HW) return fail(LI_ERR_SHAPE, "src0 length %lld is not a multiple of LH*LW=%lld", (long long)L, (long long)HW);
  const int64_t src_frames = L / HW;
  if (!frame_ids && grid.T > src_frames)
    return fail(LI_ERR_SHAPE, "grid.T=%d exceeds the %lld frames of src0", grid.T, (long long)src_frames);
  B_out = B;
  H_out = H;
  memset(&a, 0, sizeof(a));
  a.bs = grid.tt * grid.th * grid.tw;
  a.T = grid.T; a.LH = grid.LH; a.LW = grid.LW; a.tt = grid.tt; a.th = grid.th; a.tw = grid.tw;
  a.nh = (int)ceil_div(grid.LH, grid.th); a.nw = (int)ceil_div(grid.LW, grid.tw);
  nblk = ceil_div(grid.T, grid.tt) * a.nh * a.nw;
  a.H = (int)H; a.D = (int)D; a.dtype = dtype; a.CH = (int)(D * dtype_size(dtype) / 16);
  a.src_frames = (int)src_frames; a.frame_ids = frame_ids; a.flat = 0;
  a.nstreams = src1 ? 2 : 1;
  a.src[0] = static_cast<const uint8_t*>(src0->data);
  a.s_b[0] = src0->stride[0]; a.s_h[0] = src0->stride[1]; a.s_l[0] = src0->stride[2];
  if (src1) {
    if (li_status st = check_vec_view(src1->data, src1->stride, 4, src1->dtype, D, "src1")) return st;
    for (int i = 0; i < 4; ++i)
      if (src1->shape[i] != src0->shape[i]) return fail(LI_ERR_SHAPE, "src1 shape differs from src0");
    if (src1->dtype != dtype) return fail(LI_ERR_INVALID_ARG, "src1 dtype differs from src0");
    a.src[1] = static_cast<const uint8_t*>(src1->data);
    a.s_b[1] = src1->stride[0]; a.s_h[1] = src1->stride[1]; a.s_l[1] = src1->stride[2];
  }
  if (8 * a.CH * a.nstreams > 512) return fail(LI_ERR_UNSUPPORTED, "D too large for the tiling kernel");
  a.dst_off = dst_block_offset;
  a.pool_off = pool_block_offset;
  if (li_status st = fill_dst(a, 0, dst0, B, H, D, dtype, nblk + dst_block_offset, "dst0")) return st;
  if (li_status st = fill_dst(a, 1, dst1, B, H, D, dtype, nblk + dst_block_offset, "dst1")) return st;
  if (pool) {
    if (li_status st = check_vec_view(pool->data, pool->stride, 4, pool->dtype, D, "pool")) return st;
    if (pool->dtype != dtype) return fail(LI_ERR_INVALID_ARG, "pool dtype differs from the source");
    if (pool->shape[0] != B || pool->shape[1] != H || pool->shape[3] != D ||
        pool->shape[2] < nblk + pool_block_offset)
      return fail(LI_ERR_SHAPE, "pool: expected [B,H,>=%lld,D]", (long long)(nblk + pool_block_offset));
    a.pool = static_cast<uint8_t*>(pool->data);
    a.p_b = pool->stride[0]; a.p_h = pool->stride[1]; a.p_n = pool->stride[2];
  }
  if (normalize && !pool) return fail(LI_ERR_INVALID_ARG, "normalised pooling needs a pool output");
  if (!dst0 && !pool && !dst1) *empty = true;
  a.normalize = normalize;
  a.eps = dtype == LI_DTYPE_FP32 ? 1e-12f
        : dtype == LI_DTYPE_BF16 ? __bfloat162float(__float2bfloat16_rn(1e-12f))
                                 : __half2float(__float2half_rn(1e-12f));
  return LI_OK;
}

li_status tile_pool_impl(const li_view4* src0, const li_view4* src1, const int32_t* frame_ids, li_grid3d grid,
                         li_view5* dst0, li_view5* dst1, int64_t dst_block_offset, li_view4* pool,
                         int64_t pool_block_offset, int normalize, void* stream) {
  TileArgs a;
  int64_t nblk = 0, B = 0, H = 0;
  bool empty = false;
  if (li_status st = prepare_tile(src0, src1, frame_ids, grid, dst0, dst1, dst_block_offset, pool, pool_block_offset,
                                  normalize, a, nblk, B, H, &empty))
    return st;
  if (empty) return LI_OK;
  return launch_tile(a, nblk, B, H, stream);
}

size_t tile_smem(const TileArgs& a) { return (size_t)8 * a.D * 8 + (size_t)a.bs * 4 + (size_t)a.D * 4; }
}  // namespace
}  // namespace li

extern "C" li_status li_tile_pool(const li_view4* src0, const li_view4* src1, const int32_t* frame_ids,
                                  li_grid3d grid, li_view5* dst0, li_view5* dst1,
                                  int64_t dst_block_offset, li_view4* pool, int64_t pool_block_offset,
                                  void* stream) {
  return tile_pool_impl(src0, src1, frame_ids, grid, dst0, dst1, dst_block_offset, pool, pool_block_offset, 0,
                        stream);
}

extern "C" li_status li_pool_blocks(const li_view4* src, const int32_t* frame_ids, li_grid3d grid, li_view4* pool,
                                    int64_t pool_block_offset, int32_t normalized, void* stream) {
  return tile_pool_impl(src, nullptr, frame_ids, grid, nullptr, nullptr, 0, pool, pool_block_offset,
                        normalized ? 1 : 0, stream);
}

extern "C" li_status li_pool_blocks_multi(const li_pool_job* jobs, int32_t n_jobs, void* stream) {
  if (!jobs || n_jobs < 1 || n_jobs > kMaxPoolJobs)
    return fail(LI_ERR_INVALID_ARG, "1 to %d pooling jobs are required (got %d)", kMaxPoolJobs, n_jobs);
  TileMulti m;
  memset(&m, 0, sizeof(m));
  size_t smem = 0;
  int64_t total = 0;
  for (int j = 0; j < n_jobs; ++j) {
    const li_pool_job& jb = jobs[j];
    if (!jb.pool) return fail(LI_ERR_INVALID_ARG, "job %d: pool is required", j);
    int64_t nblk = 0, B = 0, H = 0;
    bool empty = false;
    if (li_status st = prepare_tile(jb.src, nullptr, jb.frame_ids, jb.grid, nullptr, nullptr, 0, jb.pool,
                                    jb.pool_block_offset, jb.normalized ? 1 : 0, m.job[m.n], nblk, B, H, &empty))
      return st;
    if (m.n > 0 && (m.job[m.n].dtype != m.job[0].dtype || m.job[m.n].CH != m.job[0].CH))
      return fail(LI_ERR_INVALID_ARG, "job %d: every job must share the dtype and head dim of job 0", j);
    if (nblk * B * H == 0) continue;
    if (B * H > 65535) return fail(LI_ERR_SHAPE, "job %d: too many (batch, head) pairs", j);
    m.start[m.n] = total;
    m.nblk[m.n] = nblk;
    total += nblk * B * H;
    smem = std::max(smem, tile_smem(m.job[m.n]));
    ++m.n;
  }
  if (m.n == 0) return LI_OK;
  m.start[m.n] = total;
  if (total > 2147483647) return fail(LI_ERR_SHAPE, "grid too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 block(8 * m.job[0].CH);
  const unsigned grid = (unsigned)total;
  if (m.job[0].dtype == LI_DTYPE_BF16) tile_pool_multi_kernel<LI_DTYPE_BF16><<<grid, block, smem, st>>>(m);
  else if (m.job[0].dtype == LI_DTYPE_FP16) tile_pool_multi_kernel<LI_DTYPE_FP16><<<grid, block, smem, st>>>(m);
  else tile_pool_multi_kernel<LI_DTYPE_FP32><<<grid, block, smem, st>>>(m);
  return launched("tile_pool_multi_kernel launch");
}

extern "C" li_status li_text_blocks(const li_view4* src0, const li_view4* src1, int32_t bs,
                                    li_view5* dst0, li_view5* dst1, void* stream) {
  if (!src0 || !dst0) return fail(LI_ERR_INVALID_ARG, "src0 and dst0 are required");
  if ((src1 == nullptr) != (dst1 == nullptr)) return fail(LI_ERR_INVALID_ARG, "dst1 must be given iff src1 is");
  if (bs <= 0 || bs % 8 || bs > kMaxBS) return fail(LI_ERR_UNSUPPORTED, "block size %d", bs);
  const int64_t B = src0->shape[0], H = src0->shape[1], N = src0->shape[2], D = src0->shape[3];
  if (N == 0) return LI_OK;
  const int dtype = src0->dtype;
  if (li_status st = check_vec_view(src0->data, src0->stride, 4, dtype, D, "src0")) return st;
  TileArgs a;
  memset(&a, 0, sizeof(a));
  a.flat = 1; a.n_tokens = (int)N; a.bs = bs; a.H = (int)H; a.D = (int)D; a.dtype = dtype;
  a.CH = (int)(D * dtype_size(dtype) / 16);
  a.nstreams = src1 ? 2 : 1;
  a.src[0] = static_cast<const uint8_t*>(src0->data);
  a.s_b[0] = src0->stride[0]; a.s_h[0] = src0->stride[1]; a.s_l[0] = src0->stride[2];
  if (src1) {
    if (li_status st = check_vec_view(src1->data, src1->stride, 4, src1->dtype, D, "src1")) return st;
    for (int i = 0; i < 4; ++i)
      if (src1->shape[i] != src0->shape[i]) return fail(LI_ERR_SHAPE, "src1 shape differs from src0");
    a.src[1] = static_cast<const uint8_t*>(src1->data);
    a.s_b[1] = src1->stride[0]; a.s_h[1] = src1->stride[1]; a.s_l[1] = src1->stride[2];
  }
  if (8 * a.CH * a.nstreams > 512) return fail(LI_ERR_UNSUPPORTED, "D too large for the tiling kernel");
  const int64_t nblk = ceil_div(N, bs);
  if (li_status st = fill_dst(a, 0, dst0, B, H, D, dtype, nblk, "dst0")) return st;
  if (li_status st = fill_dst(a, 1, dst1, B, H, D, dtype, nblk, "dst1")) return st;
  return launch_tile(a, nblk, B, H, stream);
}

extern "C" li_status li_untile(const li_view5* src, li_grid3d grid, li_view4* dst, void* stream) {
  if (!src || !dst) return fail(LI_ERR_INVALID_ARG, "src and dst are required");
  if (li_status st = check_grid(grid)) return st;
  const int64_t B = dst->shape[0], H = dst->shape[1], L = dst->shape[2], D = dst->shape[3];
  const int dtype = dst->dtype;
  if (li_status st = check_vec_view(dst->data, dst->stride, 4, dtype, D, "dst")) return st;
  if (li_status st = check_vec_view(src->data, src->stride, 5, src->dtype, D, "src")) return st;
  if (src->dtype != dtype) return fail(LI_ERR_INVALID_ARG, "src dtype differs from dst");
  const int bs = grid.tt * grid.th * grid.tw;
  const int nh = (int)ceil_div(grid.LH, grid.th), nw = (int)ceil_div(grid.LW, grid.tw);
  const int64_t nblk = ceil_div(grid.T, grid.tt) * nh * nw;
  if (L < (int64_t)grid.T * grid.LH * grid.LW) return fail(LI_ERR_SHAPE, "dst shorter than T*LH*LW");
  if (src->shape[0] != B || src->shape[1] != H || src->shape[2] < nblk || src->shape[3] != bs || src->shape[4] != D)
    return fail(LI_ERR_SHAPE, "src: expected [B,H,>=%lld,%d,D]", (long long)nblk, bs);
  UntileArgs a;
  memset(&a, 0, sizeof(a));
  a.src = static_cast<const uint8_t*>(src->data);
  a.s_b = src->stride[0]; a.s_h = src->stride[1]; a.s_n = src->stride[2]; a.s_r = src->stride[3];
  a.dst = static_cast<uint8_t*>(dst->data);
  a.d_b = dst->stride[0]; a.d_h = dst->stride[1]; a.d_l = dst->stride[2];
  a.T = grid.T; a.LH = grid.LH; a.LW = grid.LW; a.tt = grid.tt; a.th = grid.th; a.tw = grid.tw;
  a.nh = nh; a.nw = nw; a.H = (int)H; a.bs = bs; a.dtype = dtype;
  a.CH = (int)(D * dtype_size(dtype) / 16);
  if (8 * a.CH > 1024) return fail(LI_ERR_UNSUPPORTED, "D too large for the untile kernel");
  if (nblk == 0 || B * H == 0) return LI_OK;
  untile_kernel<<<dim3((unsigned)nblk, (unsigned)(B * H)), dim3(8 * a.CH), 0,
                  static_cast<cudaStream_t>(stream)>>>(a);
  return launched("untile_kernel launch");
}

extern "C" li_status li_gather_frames(const li_view4* src, const int32_t* frame_ids, int32_t n_frames,
                                      int32_t frame_tokens, li_view4* dst, uint32_t* err_word,
                                      void* stream) {
  if (!src || !dst || !frame_ids) return fail(LI_ERR_INVALID_ARG, "src, dst and frame_ids are required");
  if (n_frames < 0 || frame_tokens <= 0) return fail(LI_ERR_SHAPE, "bad frame counts");
  const int64_t B = src->shape[0], H = src->shape[1], L = src->shape[2], D = src->shape[3];
  const int dtype = src->dtype;
  if (li_status st = check_vec_view(src->data, src->stride, 4, dtype, D, "src")) return st;
  if (li_status st = check_vec_view(dst->data, dst->stride, 4, dst->dtype, D, "dst")) return st;
  if (dst->dtype != dtype) return fail(LI_ERR_INVALID_ARG, "dst dtype differs from src");
  if (L % frame_tokens) return fail(LI_ERR_SHAPE, "src length is not a multiple of frame_tokens");
  if (dst->shape[0] != B || dst->shape[1] != H || dst->shape[3] != D ||
      dst->shape[2] < (int64_t)n_frames * frame_tokens)
    return fail(LI_ERR_SHAPE, "dst: expected [B,H,>=%lld,D]", (long long)n_frames * frame_tokens);
  GatherArgs a;
  memset(&a, 0, sizeof(a));
  a.src = static_cast<const uint8_t*>(src->data);
  a.s_b = src->stride[0]; a.s_h = src->stride[1]; a.s_l = src->stride[2];
  a.dst = static_cast<uint8_t*>(dst->data);
  a.d_b = dst->stride[0]; a.d_h = dst->stride[1]; a.d_l = dst->stride[2];
  a.frame_ids = frame_ids; a.err = err_word;
  a.src_frames = (int)(L / frame_tokens); a.frame_tokens = frame_tokens; a.H = (int)H;
  a.dtype = dtype; a.CH = (int)(D * dtype_size(dtype) / 16);
  if (n_frames == 0 || B * H == 0) return LI_OK;
  const int64_t pieces = ceil_div(frame_tokens, kGatherRows);
  if ((int64_t)n_frames * pieces > 2147483647 || B * H > 65535) return fail(LI_ERR_SHAPE, "grid too large");
  gather_frames_kernel<<<dim3((unsigned)(n_frames * pieces), (unsigned)(B * H)), dim3(256), 0,
                         static_cast<cudaStream_t>(stream)>>>(a);
  return launched("gather_frames_kernel launch");
}
