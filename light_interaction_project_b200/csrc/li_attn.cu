// Block-sparse attention forward for sm_100a: TMA + tcgen05 + TMEM.
//
// One CTA per SM computes one query block (bs rows, padded to the 128-row MMA
// tile) of one (b, h) against the key blocks in its index list. The list is
// split into two independent online-softmax chains (even and odd positions),
// so the tensor core works on one chain while the other chain's softmax runs;
// a single MMA issuer serves both chains in list order, which keeps the two
// softmaxes taking turns (see the MMA issuer below).
// Twelve warps (384 threads):
//   warps 0-3 / 4-7  softmax of chain 0 / 1, then the epilogue — thread t of
//                    the warpgroup owns query row t, which is TMEM lane t;
//   warp 8           MMA issuer of both chains (one elected lane) and TMEM
//                    allocator;
//   warp 9           TMA producer of Q (once) and of every listed K_j;
//   warp 10          TMA producer of every listed V_j;
//   warp 11          no work: it completes the register donor warpgroup.
// TMEM (all 512 columns): S_0 at 0, S_1 at 128, O_0 at 256, O_1 at 384. The
// softmax writes P as packed 16-bit pairs over the first bs/2 columns of its
// chain's S, and the PV product reads it from there as the TMEM A operand (TS
// form), so P never touches shared memory.
//
// Chain c, block j:  MMA  S_c = Q K_j^T             -> commit k_empty, s_full
//                    SM   row max, lazy O_c rescale, P = exp2(S*c - m)
//                    MMA  O_c (+)= P V_j            -> commit v_empty
// The row max is only moved (and O rescaled) when it grows by more than 8 in
// log2 units; otherwise the stale max is kept (P <= 2^8), which leaves O/l
// exact. The K and V producers refill a ring stage as soon as the MMA that read
// it completes; each walks the block list 32 entries at a time from registers,
// with the next 32 entries already loading, so no copy waits on an index load.
// The row arithmetic uses packed f32x2 ops.
//
// Operands come straight from the caller's layout through 5-D tensor maps
// (d, w, h, t, b*h): a 3D (tt, th, tw) block of a raster tensor is one box, and
// TMA fills coordinates past the grid edge with zeros — exactly the zero
// padding of the tiled layout. The epilogue stores O through the same kind of
// map, and TMA drops the rows that fall outside the tensor (untiling for free).
//
// Every mbarrier wait is bounded (kTimeoutNs); on expiry the CTA records
// LI_DEVERR_TIMEOUT, drains its own copies and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstring>
#include <mutex>
#include <algorithm>

#include "li_common.cuh"

namespace li {
namespace attn {

constexpr int kMaxMaps = 4;
constexpr int kThreads = 384;  // 8 softmax warps, MMA warp, 2 TMA warps, 1 idle warp
constexpr int kWarpMMA = 8, kWarpTMAK = 9, kWarpTMAV = 10;  // warp 11: register donor only
// K and V ring stages (a third stage of either measured no faster).
constexpr int kRingK = 2, kRingV = 2;
// Registers per thread: at launch (65536 / 384, rounded down to a multiple of
// 8), and after the warpgroup split (setmaxnreg). The split never asks for more
// than the launch holds: 2*128*216 + 128*56 = 62464 <= 384*168 = 64512.
constexpr int kRegsLaunch = 168, kRegsSoftmax = 216, kRegsIssue = 56;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsIssue <= kThreads * kRegsLaunch, "register split");
constexpr uint64_t kTimeoutNs = 1000000000ull;  // 1 s per wait
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 256;  // S_0, S_1 at 0 and 128; O_0, O_1 at 256 and 384

struct __align__(64) Params {
  CUtensorMap q_map[kMaxMaps];
  CUtensorMap k_map[kMaxMaps];
  CUtensorMap v_map[kMaxMaps];
  CUtensorMap kt_map[kMaxMaps];
  CUtensorMap vt_map[kMaxMaps];
  CUtensorMap o_map[kMaxMaps];
  const int32_t* idx;
  int64_t i_b, i_h, i_q, i_s;
  const int32_t* cnt;
  int64_t c_b, c_h, c_q;
  float* lse;
  int64_t lse_len;
  uint32_t* err;
  float scale_log2;
  int32_t H, b0, per_batch;
  int32_t q_raster, kv_raster;
  int32_t q_nh, q_nw, q_tt, q_th, q_tw;
  int32_t k_nh, k_nw, k_tt, k_th, k_tw;
  int32_t ntxt, n_kv, nq;
  int32_t smax;  // index-row width: counts are clamped to it
  // Tail split. The 1-D grid lists the launch's query tiles t = (bl*H + h)*nq + qi;
  // CTAs u < n_whole take tile u whole and store it. The remaining tiles are
  // cut into nsplit pieces each: CTA u >= n_whole takes piece v = u - n_whole,
  // i.e. list entries [S*sp/nsplit, S*(sp+1)/nsplit) of tile n_whole + v/nsplit
  // (sp = v % nsplit), and writes its unnormalised fp32 partial (O at
  // part + v*128*D; m, then l, after all part_units O blocks) for
  // attn_combine_kernel.
  int64_t n_whole;
  int32_t nsplit;
  float* part;
  int64_t part_units;
  // Blocks of 256 tokens run as two 128-row sub-blocks (sub = 2, else 1). A
  // sub-block's TMA box halves one tile dimension: c[*_split] of sub-block s is
  // the block's origin + s * *_ext (for row layouts: split 1, ext = rows).
  int32_t sub, q_split, q_ext, k_split, k_ext;
};

// ------------------------------- PTX helpers -------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait. Returns false when the CTA is aborting (another warp timed
// out) or this wait ran past kTimeoutNs (then it raises the abort itself).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                       uint32_t* err, bool honour_abort = true) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = gtimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try(bar, parity)) return true;
    if ((it & 7) == 0) {
      if (honour_abort && *abort_flag) return false;
      if (gtimer() - t0 > kTimeoutNs) {
        *abort_flag = 1;
        if (err) atomicOr(err, (unsigned)LI_DEVERR_TIMEOUT);
        return false;
      }
    }
  }
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, const int c[5], uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]), "r"(c[4]), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_store_5d(const CUtensorMap* map, uint32_t src, const int c[5]) {
  asm volatile(
      "cp.async.bulk.tensor.5d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4, %5}], [%6];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]), "r"(c[4]), "r"(src)
      : "memory");
}
__device__ __forceinline__ void tma_store_commit_and_drain() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(ncols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Packed fp32 pair arithmetic (one instruction for two lanes of work).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <bool F16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t r;
  if (F16) asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 layout: start>>4
// [0,14), LBO>>4 [16,30), SBO>>4 [32,46), version 1 at bit 46, swizzle 2 at [61,64)).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16 with fp32 accumulate.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool f16, bool b_mn_major) {
  return (1u << 4) | ((f16 ? 0u : 1u) << 7) | ((f16 ? 0u : 1u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// --------------------------------- kernel ----------------------------------
template <int D, int BS>
struct Smem {
  static constexpr int kHalves = D / 64;
  // K and V ring stages: a K stage is refilled once the S MMA that read it has
  // completed, a V stage once its PV MMA has.
  static constexpr int kNK = kRingK, kNV = kRingV;
  static constexpr int kQHalf = 128 * 128;  // 128 rows of 128 bytes
  static constexpr int kKVHalf = BS * 128;
  static constexpr int kKVTile = kHalves * kKVHalf;
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kHalves * kQHalf;
  static constexpr int kOffV = kOffK + kNK * kKVTile;
  // The epilogue's per-row (m, l) of both chains (2 KB) reuses the K ring: it is
  // written only after every MMA of the tile has completed, so every K load has
  // landed and been read.
  static constexpr int kOffX = kOffK;
  static_assert(kNK * kKVTile >= 2 * 2 * 128 * 4, "K ring holds the epilogue's (m, l)");
  static constexpr int kOffBar = kOffV + kNV * kKVTile;
  // Barrier area: q | k_full[kNK] k_empty[kNK] | v_full[kNV] v_empty[kNV] |
  // s_full[2] | o_full[2] | xs | st, then the TMEM base address and the abort flag.
  static constexpr int kBarKF = 8, kBarKE = kBarKF + 8 * kNK, kBarVF = kBarKE + 8 * kNK;
  static constexpr int kBarVE = kBarVF + 8 * kNV, kBarS = kBarVE + 8 * kNV, kBarO = kBarS + 16;
  static constexpr int kBarXS = kBarO + 16, kBarST = kBarXS + 8, kSlot = kBarST + 8, kAbort = kSlot + 4;
  static_assert(kAbort + 4 <= 256, "barrier area");
  static constexpr int kBytes = kOffBar + 256 + 1024;  // + alignment slack
  static_assert(kBytes <= 227 * 1024, "shared memory per CTA");
  static constexpr uint32_t kTileBytes = (uint32_t)kKVTile;
};

__device__ __forceinline__ void block_coords(int raster, int blk, int bsz, int nh, int nw, int tt, int th, int tw,
                                             int w, int c[5]) {
  if (raster) {
    const int cw = blk % nw, rem = blk / nw, ch = rem % nh, ct = rem / nh;
    c[1] = cw * tw; c[2] = ch * th; c[3] = ct * tt;
  } else {
    c[1] = blk * bsz; c[2] = 0; c[3] = 0;
  }
  c[0] = 0;
  c[4] = w;
}

// Row of the full (256-token) query block that row r of sub-block qs is; the
// identity without sub-blocks. Raster sub-blocks halve dimension q_split.
__device__ __forceinline__ int full_block_row(const Params& p, int r, int qs, int bsk) {
  if (p.sub == 1) return r;
  if (!p.q_raster) return qs * bsk + r;
  int tw = p.q_tw, th = p.q_th, tt = p.q_tt;
  if (p.q_split == 1) tw /= 2;
  else if (p.q_split == 2) th /= 2;
  else tt /= 2;
  int ow = r % tw, rr = r / tw, oh = rr % th, ot = rr / th;
  if (p.q_split == 1) ow += qs * tw;
  else if (p.q_split == 2) oh += qs * th;
  else ot += qs * tt;
  return (ot * p.q_th + oh) * p.q_tw + ow;
}

// Named barrier over one chain's 4 softmax warps and the MMA warp. Every
// participant executes it exactly once per block of the chain (work is
// skipped, never the barrier, after an abort), so counts always match.
__device__ __forceinline__ void chain_sync(int chain) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + chain), "r"(160) : "memory");
}

// One TMA producer warp: loads tile j of every listed block (both sub-blocks of
// a 256-token block, in order) into a ring of NST stages (full barrier
// full0 + 8*stage, empty barrier empty0 + 8*stage). The
// whole warp walks the list: lane l holds entry base + l of the current 32
// entries, and the next 32 are already loading, so an index load never stands
// between two copies; lane 0 waits for the stage and issues the copy. After an
// abort, lane 0 drains the copies it issued (and, for the K producer, Q's)
// before the CTA's shared memory is released.
template <int NST, int BS>
__device__ __forceinline__ void produce(const Params& p, const int32_t* irow, int S, int lane, int wc, int mi,
                                        uint32_t ring, uint32_t tile_bytes, uint32_t half_bytes, int halves,
                                        uint32_t full0, uint32_t empty0, const CUtensorMap* vis_maps,
                                        const CUtensorMap* txt_maps, volatile int* abort_flag, uint32_t bar_q) {
  int32_t cur = lane < S ? irow[(int64_t)lane * p.i_s] : 0;
  int32_t nxt = 32 + lane < S ? irow[(int64_t)(32 + lane) * p.i_s] : 0;
  int issued = 0, jx = 0;  // jx: (sub-)blocks handed to the ring so far
  bool go = true;
  for (int j = 0; j < S && go; ++j) {
    if (j > 0 && (j & 31) == 0) {
      cur = nxt;
      nxt = j + 32 + lane < S ? irow[(int64_t)(j + 32 + lane) * p.i_s] : 0;
    }
    const int blk0 = __shfl_sync(0xFFFFFFFFu, cur, j & 31);
    for (int sb = 0; sb < p.sub; ++sb, ++jx) {
      int ok = 1;
      if (lane == 0) {
        int blk = blk0;
        if (blk < 0 || blk >= p.n_kv) {
          if (p.err) atomicOr(p.err, (unsigned)LI_DEVERR_BAD_INDEX);
          blk = 0;
        }
        int c[5];
        const CUtensorMap* m;
        if (p.kv_raster && blk < p.ntxt) {
          block_coords(0, blk, BS * p.sub, 1, 1, 1, 1, 1, wc, c);
          c[1] += sb * BS;
          m = &txt_maps[mi];
        } else {
          block_coords(p.kv_raster, p.kv_raster ? blk - p.ntxt : blk, BS * p.sub, p.k_nh, p.k_nw, p.k_tt,
                       p.k_th, p.k_tw, wc, c);
          c[p.k_split] += sb * p.k_ext;
          m = &vis_maps[mi];
        }
        const int st = jx % NST;
        if (jx >= NST && !mbar_wait(empty0 + 8 * st, ((jx / NST) - 1) & 1, abort_flag, p.err)) {
          ok = 0;
        } else {
          mbar_expect_tx(full0 + 8 * st, tile_bytes);
          for (int hf = 0; hf < halves; ++hf) {
            c[0] = 64 * hf;
            tma_load_5d(ring + st * tile_bytes + hf * half_bytes, m, c, full0 + 8 * st);
          }
          issued = jx + 1;
        }
      }
      if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) {
        go = false;
        break;
      }
    }
  }
  if (lane == 0 && *abort_flag) {
    if (bar_q) mbar_wait(bar_q, 0, abort_flag, nullptr, false);
    for (int j = issued - NST; j < issued; ++j)
      if (j >= 0) mbar_wait(full0 + 8 * (j % NST), (j / NST) & 1, abort_flag, nullptr, false);
  }
}

template <int D, int BS, bool F16>
__global__ void __launch_bounds__(kThreads, 1) attn_fwd_kernel(const __grid_constant__ Params p) {
  using L = Smem<D, BS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t cta = blockIdx.x;
  int64_t tile = cta, piece = 0;
  int sp = 0, ns = 1;
  if (cta >= p.n_whole) {
    piece = cta - p.n_whole;
    tile = p.n_whole + piece / p.nsplit;
    sp = (int)(piece % p.nsplit);
    ns = p.nsplit;
  }
  const int64_t nqt = (int64_t)p.nq * p.sub;  // query tiles per (b, h)
  const int qt = (int)(tile % nqt), qi = qt / p.sub, qs = qt % p.sub;
  const int bl = (int)(tile / nqt) / p.H, h = (int)(tile / nqt) % p.H;
  const int b = p.b0 + bl;
  const int mi = p.per_batch ? bl : 0;
  const int wc = p.per_batch ? h : b * p.H + h;

  const uint32_t bar0 = sb + L::kOffBar;
  const uint32_t bar_q = bar0;
  auto bar_kf = [&](int s) { return bar0 + L::kBarKF + 8 * s; };
  auto bar_ke = [&](int s) { return bar0 + L::kBarKE + 8 * s; };
  auto bar_vf = [&](int s) { return bar0 + L::kBarVF + 8 * s; };
  auto bar_ve = [&](int s) { return bar0 + L::kBarVE + 8 * s; };
  auto bar_s = [&](int c) { return bar0 + L::kBarS + 8 * c; };
  auto bar_o = [&](int c) { return bar0 + L::kBarO + 8 * c; };
  const uint32_t bar_xs = bar0 + L::kBarXS, bar_st = bar0 + L::kBarST;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + L::kOffBar + L::kSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffBar + L::kAbort);
  float* xm = reinterpret_cast<float*>(smem + L::kOffX);   // [2 chains][128] row max
  float* xl = xm + 2 * 128;                                 // [2 chains][128] row sum

  const int S_raw = p.cnt[b * p.c_b + h * p.c_h + (int64_t)qi * p.c_q];
  const int S_all = S_raw < 0 ? 0 : (S_raw > p.smax ? p.smax : S_raw);
  if (S_all != S_raw && threadIdx.x == 0 && sp == 0 && p.err) atomicOr(p.err, (unsigned)LI_DEVERR_BAD_INDEX);
  const int j_lo = (int)(((int64_t)S_all * sp) / ns), j_hi = (int)(((int64_t)S_all * (sp + 1)) / ns);
  const int S = j_hi - j_lo;  // this CTA's share of the list (entries)
  const int SX = S * p.sub;   // (sub-)blocks it processes
  const int32_t* irow = p.idx + b * p.i_b + h * p.i_h + (int64_t)qi * p.i_q + (int64_t)j_lo * p.i_s;
  const bool partial = ns > 1;
  const int n_chain[2] = {(SX + 1) / 2, SX / 2};  // blocks of chain 0 (even j) and chain 1 (odd j)

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < L::kNK; ++s) { mbar_init(bar_kf(s), 1); mbar_init(bar_ke(s), 1); }
    for (int s = 0; s < L::kNV; ++s) { mbar_init(bar_vf(s), 1); mbar_init(bar_ve(s), 1); }
    for (int c = 0; c < 2; ++c) { mbar_init(bar_s(c), 1); mbar_init(bar_o(c), 1); }
    mbar_init(bar_xs, 8); mbar_init(bar_st, 8);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kWarpMMA) tmem_alloc(smem_u32(smem + L::kOffBar + L::kSlot), kTmemCols);
  if (BS < 128 && warp < 4) {
    // Query rows past the block are zero so the padded MMA rows stay finite.
    for (int hf = 0; hf < L::kHalves; ++hf) {
      uint4* z = reinterpret_cast<uint4*>(smem + L::kOffQ + hf * L::kQHalf + BS * 128);
      for (int i = threadIdx.x; i < (128 - BS) * 8; i += 128) z[i] = make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Register split: the launch gives every thread kRegsLaunch; the MMA/TMA
  // warpgroup (warps 8-11) hands most of its share to the two softmax
  // warpgroups. 2 * 128 * kRegsSoftmax + 128 * kRegsIssue <= 384 * kRegsLaunch.
  if (warp >= kWarpMMA) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsIssue));
  if (warp == kWarpTMAK || warp == kWarpTMAV) {
    // ------------------------------ producers ------------------------------
    if (S > 0) {
      if (warp == kWarpTMAK && lane == 0) {
        int c[5];
        block_coords(p.q_raster, qi, BS * p.sub, p.q_nh, p.q_nw, p.q_tt, p.q_th, p.q_tw, wc, c);
        c[p.q_split] += qs * p.q_ext;
        mbar_expect_tx(bar_q, L::kTileBytes);
        for (int hf = 0; hf < L::kHalves; ++hf) {
          c[0] = 64 * hf;
          tma_load_5d(sb + L::kOffQ + hf * L::kQHalf, &p.q_map[mi], c, bar_q);
        }
      }
      if (warp == kWarpTMAK)
        produce<L::kNK, BS>(p, irow, S, lane, wc, mi, sb + L::kOffK, L::kKVTile, L::kKVHalf, L::kHalves, bar0 + L::kBarKF,
                        bar0 + L::kBarKE, p.k_map, p.kt_map, abort_flag, bar_q);
      else
        produce<L::kNV, BS>(p, irow, S, lane, wc, mi, sb + L::kOffV, L::kKVTile, L::kKVHalf, L::kHalves, bar0 + L::kBarVF,
                        bar0 + L::kBarVE, p.v_map, p.vt_map, abort_flag, 0);
    }
  } else if (warp == kWarpMMA) {
    // ------------------ MMA issuer of both chains (one lane) ------------------
    // Chain c owns key blocks j = c, c+2, ...: S_j = Q K_j^T into TMEM S_c, then
    // (after chain c's softmax) O_c += P_j V_j. One thread issues every MMA, in
    // the order S_0, S_1, PV_0, S_2, PV_1, S_3, ...; MMAs of one thread run in
    // order, so the tensor core works on one chain while the other chain's
    // softmax runs and the two softmaxes take turns on the MUFU unit (two
    // independent issuers drift into lockstep, where both softmaxes run at once
    // and the tensor core idles meanwhile). S_{j+2}, issued after PV_j, never
    // overwrites P_j before PV_j has read it, and s_full of S_j also covers
    // PV_{j-2}.
    constexpr uint32_t idS = idesc_f16(128, BS, F16, false);
    constexpr uint32_t idPV = idesc_f16(128, D, F16, true);
    const uint64_t qd = sdesc(sb + L::kOffQ, 16, 1024);
    const uint64_t kd0 = sdesc(sb + L::kOffK, 16, 1024);
    const uint64_t vd0 = sdesc(sb + L::kOffV, L::kKVHalf, 1024);
    auto issue_s = [&](int j) {
      const int ks = j % L::kNK;
      if (!mbar_wait(bar_kf(ks), (j / L::kNK) & 1, abort_flag, p.err)) return;
      tc_fence_after();
      const uint64_t kd = kd0 + (uint64_t)((ks * L::kKVTile) >> 4);
      const uint32_t tS = tmem + kColS + (uint32_t)(j & 1) * 128;
      // A K-step moves 32 bytes along a 128-byte swizzled row, four steps per
      // 64-column half: the descriptors differ only in their start address
      // field (address >> 4, no carry: shared addresses stay below 2^18).
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        mma_ss(tS, qd + (uint64_t)(((kk >> 2) * L::kQHalf + (kk & 3) * 32) >> 4),
               kd + (uint64_t)(((kk >> 2) * L::kKVHalf + (kk & 3) * 32) >> 4), idS, kk > 0 ? 1u : 0u);
      mma_commit(bar_ke(ks));
      mma_commit(bar_s(j & 1));
    };
    if (lane == 0 && SX > 0 && mbar_wait(bar_q, 0, abort_flag, p.err)) {
      tc_fence_after();
      issue_s(0);
      if (SX > 1) issue_s(1);
    }
    for (int j = 0; j < SX; ++j) {
      const int c = j & 1;
      chain_sync(c);  // chain c's softmax has written P_j (or skipped after an abort)
      if (lane == 0 && !*abort_flag) {
        tc_fence_after();
        const int vs = j % L::kNV;
        if (mbar_wait(bar_vf(vs), (j / L::kNV) & 1, abort_flag, p.err)) {
          tc_fence_after();
          const uint64_t vd = vd0 + (uint64_t)((vs * L::kKVTile) >> 4);
          const uint32_t tS = tmem + kColS + (uint32_t)c * 128, tO = tmem + kColO + (uint32_t)c * 128;
#pragma unroll
          for (int kk = 0; kk < BS / 16; ++kk)
            mma_ts(tO, tS + kk * 8, vd + (uint64_t)((kk * 2048) >> 4), idPV, (j >= 2 || kk > 0) ? 1u : 0u);
          mma_commit(bar_ve(vs));
          if (j + 2 < SX) issue_s(j + 2);
        }
      }
      __syncwarp();
    }
    if (lane == 0 && SX > 0) {
      // Every MMA completes before O is read and TMEM is freed.
      for (int c = 0; c < 2; ++c)
        if (n_chain[c] > 0) mma_commit(bar_o(c));
      for (int c = 0; c < 2; ++c)
        if (n_chain[c] > 0) mbar_wait(bar_o(c), 0, abort_flag, p.err, false);
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    // --------------------- softmax of chain w + epilogue -----------------------
    // Thread (warp, lane) owns row = (warp & 3) * 32 + lane = TMEM lane.
    const int w = warp >> 2;
    const int nb = n_chain[w];
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_base + kColS + (uint32_t)w * 128;
    const uint32_t tO = tmem + lane_base + kColO + (uint32_t)w * 128;
    const float c2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < nb; ++i) {
      if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(bar_s(w), i & 1, abort_flag, p.err));
      if (ok) {
        tc_fence_after();
        uint32_t r[BS / 32][32];
#pragma unroll
        for (int cc = 0; cc < BS / 32; ++cc) tmem_ld32(tS + cc * 32, r[cc]);
        tmem_wait_ld();
        float mxa[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int cc = 0; cc < BS / 32; ++cc)
#pragma unroll
          for (int e = 0; e < 32; e += 8)
#pragma unroll
            for (int a = 0; a < 4; ++a)
              mxa[a] = fmax3(mxa[a], __uint_as_float(r[cc][e + 2 * a]), __uint_as_float(r[cc][e + 2 * a + 1]));
        const float mx = fmaxf(fmax3(mxa[0], mxa[1], mxa[2]), mxa[3]);
        const float m_new = fmaxf(m, mx * c2);
        // Lazy correction: move the reference max only when it grows by more
        // than 8 (log2 units); P <= 2^8 otherwise, and O/l stays exact.
        const bool need = (i > 0) && (m_new - m > 8.0f);
        const float alpha = need ? ex2(m - m_new) : 1.f;
        if (i == 0 || need) m = m_new;
        // p = 2^(s*c - m) for column pairs; P goes back over S as packed
        // 16-bit pairs.
        const float2 c2v = make_float2(c2, c2), nm = make_float2(-m, -m);
        float2 la = make_float2(0.f, 0.f), lb = make_float2(0.f, 0.f);
#pragma unroll
        for (int cc = 0; cc < BS / 32; ++cc) {
          uint32_t pk[16];
#pragma unroll
          for (int e2 = 0; e2 < 16; ++e2) {
            const float2 x =
                ffma2(make_float2(__uint_as_float(r[cc][2 * e2]), __uint_as_float(r[cc][2 * e2 + 1])), c2v, nm);
            const float2 pp = make_float2(ex2(x.x), ex2(x.y));
            if (e2 & 1) lb = fadd2(lb, pp);
            else la = fadd2(la, pp);
            pk[e2] = pack2<F16>(pp.x, pp.y);
          }
          tmem_st16(tS + cc * 16, pk);
        }
        l = l * alpha + ((la.x + la.y) + (lb.x + lb.y));
        // O_w rescale (its last PV completed before s_full of this block fired;
        // PV_j is only issued after the chain barrier below).
        if (__any_sync(0xFFFFFFFFu, need)) {
#pragma unroll
          for (int cc = 0; cc < D / 32; ++cc) {
            uint32_t o[32];
            tmem_ld32(tO + cc * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(tO + cc * 32, o);
          }
        }
        tmem_wait_st();
      }
      tc_fence_before();
      chain_sync(w);  // P_j is in TMEM: the chain's MMA warp may issue PV_j
    }
    // ---- epilogue: merge the two chains, O = (a0 O_0 + a1 O_1) / (a0 l0 + a1 l1)
    // Every MMA of both chains completes first: (m, l) go to the K ring, which
    // is free once the last S MMA has read its stage.
    for (int c = 0; c < 2; ++c)
      if (ok && n_chain[c] > 0) ok = __all_sync(0xFFFFFFFFu, mbar_wait(bar_o(c), 0, abort_flag, p.err));
    if (ok) {
      xm[w * 128 + row] = m;
      xl[w * 128 + row] = l;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_xs);
    if (ok) ok = __all_sync(0xFFFFFFFFu, mbar_wait(bar_xs, 0, abort_flag, p.err));
    tc_fence_after();
    const float m0 = xm[row], m1 = xm[128 + row], l0 = xl[row], l1 = xl[128 + row];
    const float mm = fmaxf(m0, m1);
    const float a0 = l0 > 0.f ? ex2(m0 - mm) : 0.f, a1 = l1 > 0.f ? ex2(m1 - mm) : 0.f;
    const float lt = a0 * l0 + a1 * l1;
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    // Warp-uniform: the TMEM loads below are warp-collective.
    const bool store = __all_sync(0xFFFFFFFFu, ok && !*abort_flag);
    if (partial) {
      // Unnormalised partial of this split: O = a0 O_0 + a1 O_1 relative to mm.
      const int64_t unit = piece;
      float* po = p.part + unit * 128 * D + (int64_t)row * D;
      constexpr int kOCols = D / 2;
      const uint32_t o0 = tmem + lane_base + kColO, o1 = tmem + lane_base + kColO + 128;
      if (store) {
#pragma unroll
        for (int cc = 0; cc < kOCols / 32; ++cc) {
          const int col0 = w * kOCols + cc * 32;
          uint32_t x0[32], x1[32];
          // tcgen05.ld is warp-collective: load both chains unconditionally and
          // let each lane's l decide below (a NaN row sum must not split the warp).
          tmem_ld32(o0 + col0, x0);
          tmem_ld32(o1 + col0, x1);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            float4 v;
            v.x = (l0 > 0.f ? __uint_as_float(x0[e]) * a0 : 0.f) + (l1 > 0.f ? __uint_as_float(x1[e]) * a1 : 0.f);
            v.y = (l0 > 0.f ? __uint_as_float(x0[e + 1]) * a0 : 0.f) + (l1 > 0.f ? __uint_as_float(x1[e + 1]) * a1 : 0.f);
            v.z = (l0 > 0.f ? __uint_as_float(x0[e + 2]) * a0 : 0.f) + (l1 > 0.f ? __uint_as_float(x1[e + 2]) * a1 : 0.f);
            v.w = (l0 > 0.f ? __uint_as_float(x0[e + 3]) * a0 : 0.f) + (l1 > 0.f ? __uint_as_float(x1[e + 3]) * a1 : 0.f);
            *reinterpret_cast<float4*>(po + col0 + e) = v;
          }
        }
        if (w == 0) {
          float* pml = p.part + p.part_units * 128 * D;
          pml[unit * 128 + row] = lt > 0.f ? mm : -INFINITY;
          pml[p.part_units * 128 + unit * 128 + row] = lt;
        }
      }
    } else if (store) {
      uint8_t* stage = smem + L::kOffQ;
      constexpr int kOCols = D / 2;  // this warpgroup converts O columns [w*D/2, (w+1)*D/2)
      const uint32_t o0 = tmem + lane_base + kColO, o1 = tmem + lane_base + kColO + 128;
#pragma unroll
      for (int cc = 0; cc < kOCols / 32; ++cc) {
        const int col0 = w * kOCols + cc * 32;
        uint32_t x0[32], x1[32];
        // tcgen05.ld is warp-collective: load both chains unconditionally and
        // let each lane's l decide below (a NaN row sum must not split the warp).
        tmem_ld32(o0 + col0, x0);
        tmem_ld32(o1 + col0, x1);
        tmem_wait_ld();
        const float s0 = a0 * inv, s1 = a1 * inv;
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float v0 = (l0 > 0.f ? __uint_as_float(x0[2 * e]) * s0 : 0.f) +
                           (l1 > 0.f ? __uint_as_float(x1[2 * e]) * s1 : 0.f);
          const float v1 = (l0 > 0.f ? __uint_as_float(x0[2 * e + 1]) * s0 : 0.f) +
                           (l1 > 0.f ? __uint_as_float(x1[2 * e + 1]) * s1 : 0.f);
          pk[e] = pack2<F16>(v0, v1);
        }
        const int hf = col0 / 64, ch0 = (col0 % 64) / 8;
        uint8_t* rowp = stage + hf * L::kQHalf + row * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int phys = (ch0 + q) ^ (row & 7);
          *reinterpret_cast<uint4*>(rowp + phys * 16) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      fence_proxy_async_smem();
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_st);
    if (store && !partial && threadIdx.x == 0 && mbar_wait(bar_st, 0, abort_flag, p.err) && !*abort_flag) {
      int c[5];
      block_coords(p.q_raster, qi, BS * p.sub, p.q_nh, p.q_nw, p.q_tt, p.q_th, p.q_tw, wc, c);
      c[p.q_split] += qs * p.q_ext;
      for (int hf = 0; hf < L::kHalves; ++hf) {
        c[0] = 64 * hf;
        tma_store_5d(&p.o_map[mi], sb + L::kOffQ + hf * L::kQHalf, c);
      }
      tma_store_commit_and_drain();
    }
    if (store && !partial && w == 0 && p.lse && row < BS)
      p.lse[(int64_t)(b * p.H + h) * p.lse_len + (int64_t)qi * BS * p.sub + full_block_row(p, row, qs, BS)] =
          lt > 0.f ? mm + __log2f(lt) : -INFINITY;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMMA) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}


// ------------------------- split-KV combine kernel -------------------------
// Merges the nsplit partials O_s (unnormalised, reference max m_s, row sum l_s)
// of each split tile (tile n_whole + blockIdx.x of the launch):
//   M = max m_s,  w_s = 2^(m_s - M),  O = sum w_s O_s / sum w_s l_s,
// and stores each row at its raster (or tiled) position in o. A CTA takes
// kCombRows rows: their per-piece weights go to shared memory first, then
// each thread reduces one 8-column chunk of one row, so consecutive threads
// read consecutive 32-byte pieces of the partials.
constexpr int kCombRows = 16, kCombThreads = 256, kMaxPieces = 16;
struct CombineArgs {
  const float* part;
  int64_t part_units;
  uint8_t* o;
  int64_t o_b, o_h, o_l;
  float* lse;
  int64_t lse_len;
  int64_t n_whole;
  int32_t H, b0, nq, nsplit, D, bs, f16;
  int32_t q_raster, T, LH, LW, tt, th, tw, nh, nw;
  int64_t q_len;  // tiled form: valid query rows
  int32_t sub, q_split, bsk;  // sub-blocks of a query block (rows bsk each), as in Params
};

__global__ void __launch_bounds__(kCombThreads) attn_combine_kernel(const CombineArgs a) {
  static_assert(kCombRows * kMaxPieces == kCombThreads, "one thread per (row, piece) in the weight pass");
  __shared__ float wgt[kMaxPieces][kCombRows];
  __shared__ int64_t tok_s[kCombRows];
  const int64_t tile = a.n_whole + blockIdx.x;
  const int64_t nqt = (int64_t)a.nq * a.sub;
  const int qt = (int)(tile % nqt), qi = qt / a.sub, qs = qt % a.sub;
  const int b = a.b0 + (int)(tile / nqt) / a.H, h = (int)(tile / nqt) % a.H;
  const int bh = b * a.H + h;
  const int r0 = blockIdx.y * kCombRows;
  const int64_t unit0 = (int64_t)blockIdx.x * a.nsplit;
  const float* pm = a.part + a.part_units * 128 * a.D;
  const float* pl = pm + a.part_units * 128;
  {
    // Weight pass: thread (lr, sp) holds piece sp of row r0 + lr; the 16 pieces
    // of a row are 16 adjacent lanes, reduced with shuffles.
    const int lr = threadIdx.x / kMaxPieces, sp = threadIdx.x % kMaxPieces;
    const int row = r0 + lr;
    const bool have = sp < a.nsplit;
    const float m = have ? pm[(unit0 + sp) * 128 + row] : -INFINITY;
    const float l = have ? pl[(unit0 + sp) * 128 + row] : 0.f;
    float M = l > 0.f ? m : -INFINITY;
#pragma unroll
    for (int o = kMaxPieces / 2; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    const float e = l > 0.f ? ex2(m - M) : 0.f;
    float L = e * l;
#pragma unroll
    for (int o = kMaxPieces / 2; o > 0; o >>= 1) L += __shfl_xor_sync(0xFFFFFFFFu, L, o);
    const float inv = L > 0.f ? 1.f / L : 0.f;
    wgt[sp][lr] = e * inv;
    if (sp == 0) {
      // Row of the full query block (sub-blocks halve dimension q_split).
      int frow = row;
      if (a.sub > 1) {
        if (!a.q_raster) {
          frow = qs * a.bsk + row;
        } else {
          int tw = a.tw, th = a.th, tt = a.tt;
          if (a.q_split == 1) tw /= 2;
          else if (a.q_split == 2) th /= 2;
          else tt /= 2;
          int ow = row % tw, rr = row / tw, oh = rr % th, ot = rr / th;
          if (a.q_split == 1) ow += qs * tw;
          else if (a.q_split == 2) oh += qs * th;
          else ot += qs * tt;
          frow = (ot * a.th + oh) * a.tw + ow;
        }
      }
      int64_t tok;
      if (a.q_raster) {
        const int cw = qi % a.nw, rem = qi / a.nw, ch = rem % a.nh, ct = rem / a.nh;
        const int ow = frow % a.tw, rr = frow / a.tw, oh = rr % a.th, ot = rr / a.th;
        const int t = ct * a.tt + ot, hh = ch * a.th + oh, w = cw * a.tw + ow;
        tok = (t < a.T && hh < a.LH && w < a.LW) ? ((int64_t)t * a.LH + hh) * a.LW + w : -1;
      } else {
        tok = (int64_t)qi * a.bs + frow;
        if (tok >= a.q_len) tok = -1;
      }
      tok_s[lr] = tok;
      if (a.lse && tok >= 0)
        a.lse[(int64_t)bh * a.lse_len + (int64_t)qi * a.bs + frow] = L > 0.f ? M + __log2f(L) : -INFINITY;
    }
  }
  __syncthreads();
  const int cpr = a.D / 8;  // 8-column chunks per row
  for (int i = threadIdx.x; i < kCombRows * cpr; i += kCombThreads) {
    const int lr = i / cpr, d0 = (i % cpr) * 8;
    const int64_t tok = tok_s[lr];
    if (tok < 0) continue;
    const int row = r0 + lr;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // Pieces in groups of 8: a group's 16 loads are all issued before they are
    // used (indices past nsplit re-read the last piece with weight 0; a zero
    // weight selects 0, so an unwritten partial cannot leak into the row).
    for (int g0 = 0; g0 < a.nsplit; g0 += 8) {
      float4 x[8], y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int sp = min(g0 + e, a.nsplit - 1);
        const float4* src = reinterpret_cast<const float4*>(a.part + ((unit0 + sp) * 128 + row) * a.D + d0);
        x[e] = src[0];
        y[e] = src[1];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float w = g0 + e < a.nsplit ? wgt[g0 + e][lr] : 0.f;
        const bool on = w != 0.f;
        acc[0] += on ? w * x[e].x : 0.f; acc[1] += on ? w * x[e].y : 0.f;
        acc[2] += on ? w * x[e].z : 0.f; acc[3] += on ? w * x[e].w : 0.f;
        acc[4] += on ? w * y[e].x : 0.f; acc[5] += on ? w * y[e].y : 0.f;
        acc[6] += on ? w * y[e].z : 0.f; acc[7] += on ? w * y[e].w : 0.f;
      }
    }
    uint4 v;
    if (a.f16) {
      v.x = pack2<true>(acc[0], acc[1]); v.y = pack2<true>(acc[2], acc[3]);
      v.z = pack2<true>(acc[4], acc[5]); v.w = pack2<true>(acc[6], acc[7]);
    } else {
      v.x = pack2<false>(acc[0], acc[1]); v.y = pack2<false>(acc[2], acc[3]);
      v.z = pack2<false>(acc[4], acc[5]); v.w = pack2<false>(acc[6], acc[7]);
    }
    *reinterpret_cast<uint4*>(a.o + (b * a.o_b + h * a.o_h + tok * a.o_l) * 2 + d0 * 2) = v;
  }
}

// ------------------------------ host side ----------------------------------
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Describes one operand as a 5-D tensor (d, x, y, z, w) for TMA.
struct MapSpec {
  const void* base;
  uint64_t dims[5];
  uint64_t strides[4];  // bytes, dims 1..4
  uint32_t box[5];
};

li_status encode(CUtensorMap* out, const MapSpec& s, bool f16, const char* name) {
  auto fn = get_encode();
  if (!fn) return fail(LI_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[5], strides[4];
  cuuint32_t box[5], es[5] = {1, 1, 1, 1, 1};
  for (int i = 0; i < 5; ++i) { dims[i] = s.dims[i]; box[i] = s.box[i]; }
  for (int i = 0; i < 4; ++i) {
    strides[i] = s.strides[i];
    if (strides[i] % 16 || strides[i] >= (1ull << 40))
      return fail(LI_ERR_ALIGNMENT, "%s: stride %d (%llu bytes) is not a multiple of 16 below 2^40", name, i + 1,
                  (unsigned long long)strides[i]);
  }
  for (int i = 0; i < 5; ++i)
    if (dims[i] == 0 || dims[i] > (1ull << 32)) return fail(LI_ERR_SHAPE, "%s: dim %d out of range", name, i);
  if (!aligned16(s.base)) return fail(LI_ERR_ALIGNMENT, "%s: base pointer not 16-byte aligned", name);
  CUresult r = fn(out, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5,
                  const_cast<void*>(s.base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LI_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
  return LI_OK;
}

// How the (b, h) pair is addressed: merged into one dim, or one map per batch.
struct BHPlan {
  bool merged;
  uint64_t w_dim;
  int64_t w_stride;  // elements
};

BHPlan plan_bh(const li_view4& v) {
  const int64_t B = v.shape[0], H = v.shape[1];
  BHPlan pl;
  if (B == 1) { pl.merged = true; pl.w_dim = (uint64_t)H; pl.w_stride = v.stride[1]; }
  else if (H == 1) { pl.merged = true; pl.w_dim = (uint64_t)B; pl.w_stride = v.stride[0]; }
  else if (v.stride[0] == H * v.stride[1]) { pl.merged = true; pl.w_dim = (uint64_t)(B * H); pl.w_stride = v.stride[1]; }
  else { pl.merged = false; pl.w_dim = (uint64_t)H; pl.w_stride = v.stride[1]; }
  return pl;
}

// Raster operand: (d, w, h, t, bh); box = one (tt, th, tw) block.
MapSpec raster_spec(const li_view4& v, const li_grid3d& g, const BHPlan& pl, int b, int es, int split = 0) {
  MapSpec s;
  const int64_t sl = v.stride[2] * es;
  s.base = static_cast<const uint8_t*>(v.data) + (pl.merged ? 0 : b * v.stride[0] * es);
  s.dims[0] = (uint64_t)v.shape[3]; s.dims[1] = (uint64_t)g.LW; s.dims[2] = (uint64_t)g.LH;
  s.dims[3] = (uint64_t)(v.shape[2] / ((int64_t)g.LH * g.LW)); s.dims[4] = pl.w_dim;
  s.strides[0] = (uint64_t)sl; s.strides[1] = (uint64_t)(sl * g.LW); s.strides[2] = (uint64_t)(sl * g.LW * g.LH);
  s.strides[3] = (uint64_t)(pl.w_stride * es);
  s.box[0] = 64; s.box[1] = (uint32_t)g.tw; s.box[2] = (uint32_t)g.th; s.box[3] = (uint32_t)g.tt; s.box[4] = 1;
  if (split) s.box[split] /= 2;  // one 128-row sub-block of a 256-token block
  return s;
}

// The tile dimension a 256-token block is halved along (c / box index: 1 w,
// 2 h, 3 t; the slowest even one), and the half extent.
void sub_split(const li_grid3d& g, int32_t* split, int32_t* ext) {
  if (g.tt % 2 == 0) { *split = 3; *ext = g.tt / 2; }
  else if (g.th % 2 == 0) { *split = 2; *ext = g.th / 2; }
  else { *split = 1; *ext = g.tw / 2; }
}

// Row operand: (d, rows, 1, 1, bh); box = bs consecutive rows.
MapSpec rows_spec(const li_view4& v, int bs, const BHPlan& pl, int b, int es) {
  MapSpec s;
  const int64_t sl = v.stride[2] * es;
  s.base = static_cast<const uint8_t*>(v.data) + (pl.merged ? 0 : b * v.stride[0] * es);
  s.dims[0] = (uint64_t)v.shape[3]; s.dims[1] = (uint64_t)v.shape[2]; s.dims[2] = 1; s.dims[3] = 1;
  s.dims[4] = pl.w_dim;
  s.strides[0] = (uint64_t)sl;
  s.strides[1] = (uint64_t)(sl * v.shape[2] + 15) / 16 * 16;
  s.strides[2] = s.strides[1];
  s.strides[3] = (uint64_t)(pl.w_stride * es);
  s.box[0] = 64; s.box[1] = (uint32_t)bs; s.box[2] = 1; s.box[3] = 1; s.box[4] = 1;
  return s;
}

using KernelFn = void (*)(Params);

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Tail split of one launch. At one CTA per SM, `tiles` equal query tiles run
// as W = tiles / SMs full waves and a last wave of r = tiles % SMs tiles that
// leaves the other SMs idle for a whole tile's time. Each of those r tiles is
// cut into s list pieces instead (fp32 partials merged by the combine kernel).
// s minimises the estimated finish time, in block iterations of a list of
// `smax` blocks:  W (S + 2) + ceil(r s / SMs) (S / s + 8) + 10  (a piece pays a
// prologue and a partial store; the combine pass runs after the launch), and
// is used only when that beats the unsplit (W + 1) (S + 2) by 3%.
struct TailPlan {
  int64_t n_whole;  // tiles run whole (the first n_whole of the launch)
  int32_t pieces;   // pieces per remaining tile (1: no split)
};

TailPlan tail_plan(int64_t tiles, int64_t smax) {
  TailPlan tp{tiles, 1};
  const int64_t sms = sm_count();
  if (tiles <= 0 || smax < 8) return tp;
  const int64_t W = tiles / sms, r = tiles % sms;
  if (r == 0) return tp;
  const double S = (double)smax;
  const double whole = (double)(W + 1) * (S + 2.0);
  double best = whole;
  int best_s = 1;
  for (int s = 2; s <= kMaxPieces && S / s >= 4.0; ++s) {
    const double waves = (double)((r * s + sms - 1) / sms);
    const double c = (double)W * (S + 2.0) + waves * (S / s + 8.0) + 10.0;
    if (c < best) { best = c; best_s = s; }
  }
  if (best_s > 1 && best < 0.97 * whole) { tp.n_whole = tiles - r; tp.pieces = best_s; }
  return tp;
}

// Partial slots of a plan: (tiles - n_whole) * pieces.
int64_t plan_units(int64_t tiles, const TailPlan& tp) { return tp.pieces > 1 ? (tiles - tp.n_whole) * tp.pieces : 0; }

int64_t workspace_bytes(int64_t units, int64_t D) { return units * 128 * (D + 2) * 4; }

// Partial slots a call may need: one launch covers all B batches or, when the
// operands' batch and head strides do not merge, at most kMaxMaps of them.
int64_t call_units(int64_t B, int64_t H, int64_t nq, int64_t smax, int sub) {
  int64_t u = 0;
  for (int64_t nb : {B, std::min<int64_t>(B, kMaxMaps), B % kMaxMaps}) {
    const int64_t t = nb * H * nq * sub;
    u = std::max(u, plan_units(t, tail_plan(t, smax * sub)));
  }
  return u;
}

template <int D, int BS, bool F16>
li_status launch_t(const Params& prm, dim3 grid, cudaStream_t stream) {
  using L = Smem<D, BS>;
  static std::atomic<uint64_t> configured{0};
  if (li_status st = once_per_device(configured, [] {
        return cuda_status(cudaFuncSetAttribute(attn_fwd_kernel<D, BS, F16>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes),
                           "attention smem attribute");
      })) return st;
  attn_fwd_kernel<D, BS, F16><<<grid, kThreads, L::kBytes, stream>>>(prm);
  return launched("attention kernel launch");
}

li_status launch(int D, int BS, bool f16, const Params& prm, dim3 grid, cudaStream_t s) {
  if (D == 128 && BS == 128) return f16 ? launch_t<128, 128, true>(prm, grid, s) : launch_t<128, 128, false>(prm, grid, s);
  if (D == 128 && BS == 64) return f16 ? launch_t<128, 64, true>(prm, grid, s) : launch_t<128, 64, false>(prm, grid, s);
  if (D == 64 && BS == 128) return f16 ? launch_t<64, 128, true>(prm, grid, s) : launch_t<64, 128, false>(prm, grid, s);
  if (D == 64 && BS == 64) return f16 ? launch_t<64, 64, true>(prm, grid, s) : launch_t<64, 64, false>(prm, grid, s);
  if (D == 128 && BS == 32) return f16 ? launch_t<128, 32, true>(prm, grid, s) : launch_t<128, 32, false>(prm, grid, s);
  if (D == 64 && BS == 32) return f16 ? launch_t<64, 32, true>(prm, grid, s) : launch_t<64, 32, false>(prm, grid, s);
  return fail(LI_ERR_UNSUPPORTED, "attention built for D in {64,128} and block size in {32,64,128,256} (got D=%d bs=%d)",
              D, BS);
}

li_status check_operand(const li_view4* v, const char* name, int dtype, int64_t B, int64_t H, int64_t D) {
  if (!v || !v->data) return fail(LI_ERR_INVALID_ARG, "%s is required", name);
  if (v->dtype != dtype) return fail(LI_ERR_INVALID_ARG, "%s: dtype differs from q", name);
  if (v->shape[0] != B || v->shape[1] != H || v->shape[3] != D)
    return fail(LI_ERR_SHAPE, "%s: expected [B=%lld, H=%lld, *, D=%lld]", name, (long long)B, (long long)H, (long long)D);
  if (v->stride[3] != 1) return fail(LI_ERR_STRIDE, "%s: head dim must be contiguous", name);
  if (!aligned16(v->data)) return fail(LI_ERR_ALIGNMENT, "%s: base pointer not 16-byte aligned", name);
  return LI_OK;
}

// Shared driver of both public forms.
li_status run(const li_view4* q, bool q_raster, const li_grid3d* gq, const li_view4* k, const li_view4* v,
              bool kv_raster, const li_grid3d* gk, const li_view4* kt, const li_view4* vt, int bs,
              const li_index_view* idx, float sm_scale, li_view4* o, float* lse, uint32_t* err, void* workspace,
              int64_t workspace_bytes_avail, void* stream) {
  if (!q || !q->data) return fail(LI_ERR_INVALID_ARG, "q is required");
  const int dtype = q->dtype;
  if (dtype != LI_DTYPE_BF16 && dtype != LI_DTYPE_FP16)
    return fail(LI_ERR_UNSUPPORTED, "attention runs on bf16 or fp16 operands (got dtype %d)", dtype);
  const bool f16 = dtype == LI_DTYPE_FP16;
  const int es = 2;
  const int64_t B = q->shape[0], H = q->shape[1], D = q->shape[3];
  if (D != 64 && D != 128) return fail(LI_ERR_UNSUPPORTED, "head dim %lld (built for 64 and 128)", (long long)D);
  if (bs != 32 && bs != 64 && bs != 128 && bs != 256)
    return fail(LI_ERR_UNSUPPORTED, "block size %d (built for 32, 64, 128, 256)", bs);
  // 256-token blocks run as two 128-row sub-blocks.
  const int sub = bs == 256 ? 2 : 1, bsk = bs / sub;
  for (const li_view4* t : {q, k, v, (const li_view4*)o})
    if (li_status st = check_operand(t, t == q ? "q" : t == k ? "k" : t == v ? "v" : "o", dtype, B, H, D)) return st;
  if (o->shape[2] != q->shape[2]) return fail(LI_ERR_SHAPE, "o must have q's shape");
  for (int i = 0; i < 4; ++i)
    if (k->shape[i] != v->shape[i]) return fail(LI_ERR_SHAPE, "k and v shapes differ");
  if (!idx || !idx->indices || !idx->counts) return fail(LI_ERR_INVALID_ARG, "index view required");
  if (idx->shape[0] != B || idx->shape[1] != H) return fail(LI_ERR_SHAPE, "indices: leading dims must be [B, H]");

  Params prm;
  memset(&prm, 0, sizeof(prm));
  int64_t nq, n_kv;
  int ntxt = 0;
  if (q_raster) {
    const int64_t HW = (int64_t)gq->LH * gq->LW;
    if ((int64_t)gq->tt * gq->th * gq->tw != bs) return fail(LI_ERR_SHAPE, "grid_q tile does not give bs");
    if (q->shape[2] != (int64_t)gq->T * HW) return fail(LI_ERR_SHAPE, "q length must be T*LH*LW of grid_q");
    if (gq->tw > 256 || gq->th > 256 || gq->tt > 256) return fail(LI_ERR_UNSUPPORTED, "tile dims must be <= 256");
    prm.q_nh = (int)ceil_div(gq->LH, gq->th); prm.q_nw = (int)ceil_div(gq->LW, gq->tw);
    prm.q_tt = gq->tt; prm.q_th = gq->th; prm.q_tw = gq->tw;
    nq = ceil_div(gq->T, gq->tt) * prm.q_nh * prm.q_nw;
  } else {
    nq = ceil_div(q->shape[2], bs);
  }
  if (kv_raster) {
    const int64_t HW = (int64_t)gk->LH * gk->LW;
    if ((int64_t)gk->tt * gk->th * gk->tw != bs) return fail(LI_ERR_SHAPE, "grid_k tile does not give bs");
    if (k->shape[2] != (int64_t)gk->T * HW) return fail(LI_ERR_SHAPE, "k_vis length must be T*LH*LW of grid_k");
    prm.k_nh = (int)ceil_div(gk->LH, gk->th); prm.k_nw = (int)ceil_div(gk->LW, gk->tw);
    prm.k_tt = gk->tt; prm.k_th = gk->th; prm.k_tw = gk->tw;
    if ((kt == nullptr) != (vt == nullptr)) return fail(LI_ERR_INVALID_ARG, "k_txt and v_txt go together");
    if (kt && kt->shape[2] > 0) {
      if (li_status st = check_operand(kt, "k_txt", dtype, B, H, D)) return st;
      if (li_status st = check_operand(vt, "v_txt", dtype, B, H, D)) return st;
      if (kt->shape[2] != vt->shape[2]) return fail(LI_ERR_SHAPE, "k_txt and v_txt lengths differ");
      ntxt = (int)ceil_div(kt->shape[2], bs);
    }
    n_kv = ntxt + ceil_div(gk->T, gk->tt) * prm.k_nh * prm.k_nw;
  } else {
    if (k->shape[2] % bs) return fail(LI_ERR_SHAPE, "K length (%lld) must be divisible by logical_block_size (%d)",
                                      (long long)k->shape[2], bs);
    n_kv = k->shape[2] / bs;
  }
  if (idx->shape[2] < nq) return fail(LI_ERR_SHAPE, "indices have %lld query blocks, need %lld",
                                      (long long)idx->shape[2], (long long)nq);
  if (n_kv > (1ll << 30) || nq > (1ll << 30)) return fail(LI_ERR_SHAPE, "too many blocks");
  prm.idx = idx->indices; prm.i_b = idx->stride[0]; prm.i_h = idx->stride[1]; prm.i_q = idx->stride[2]; prm.i_s = idx->stride[3];
  prm.cnt = idx->counts; prm.c_b = idx->count_stride[0]; prm.c_h = idx->count_stride[1]; prm.c_q = idx->count_stride[2];
  prm.lse = lse; prm.lse_len = nq * bs; prm.err = err;
  prm.scale_log2 = sm_scale * 1.4426950408889634f;
  prm.H = (int)H; prm.q_raster = q_raster; prm.kv_raster = kv_raster;
  prm.ntxt = ntxt; prm.n_kv = (int)n_kv; prm.nq = (int)nq;
  if (idx->shape[3] < 0 || idx->shape[3] > (1ll << 30)) return fail(LI_ERR_SHAPE, "bad index-row width");
  prm.smax = (int)idx->shape[3];
  prm.sub = sub;
  prm.q_split = 1; prm.q_ext = bsk; prm.k_split = 1; prm.k_ext = bsk;  // row layouts
  if (sub > 1 && q_raster) sub_split(*gq, &prm.q_split, &prm.q_ext);
  if (sub > 1 && kv_raster) sub_split(*gk, &prm.k_split, &prm.k_ext);
  if (nq == 0 || B * H == 0) return LI_OK;
  if (B * H * nq * sub > INT32_MAX) return fail(LI_ERR_SHAPE, "too many query tiles for one launch");

  // All operands share one (b, h) addressing plan; fall back to per-batch
  // maps when any operand's batch and head strides do not merge.
  const li_view4* ops[6] = {q, k, v, o, kt && ntxt ? kt : nullptr, vt && ntxt ? vt : nullptr};
  bool merged = true;
  for (const li_view4* t : ops)
    if (t) merged = merged && plan_bh(*t).merged && (plan_bh(*t).w_dim == plan_bh(*q).w_dim || B == 1 || H == 1);
  const int64_t chunk = merged ? B : kMaxMaps;
  for (int64_t b0 = 0; b0 < B; b0 += chunk) {
    const int64_t nb = std::min<int64_t>(chunk, B - b0);
    prm.b0 = (int)b0;
    prm.per_batch = merged ? 0 : 1;
    for (int64_t i = 0; i < (merged ? 1 : nb); ++i) {
      const int bb = (int)(b0 + i);
      auto pl = [&](const li_view4& t) {
        BHPlan x = plan_bh(t);
        if (!merged) { x.merged = false; x.w_dim = (uint64_t)H; x.w_stride = t.stride[1]; }
        return x;
      };
      li_status st;
      const int qsp = sub > 1 ? prm.q_split : 0, ksp = sub > 1 ? prm.k_split : 0;
      if (q_raster) {
        st = encode(&prm.q_map[i], raster_spec(*q, *gq, pl(*q), bb, es, qsp), f16, "q");
        if (!st) st = encode(&prm.o_map[i], raster_spec(*o, *gq, pl(*o), bb, es, qsp), f16, "o");
      } else {
        st = encode(&prm.q_map[i], rows_spec(*q, bsk, pl(*q), bb, es), f16, "q");
        if (!st) st = encode(&prm.o_map[i], rows_spec(*o, bsk, pl(*o), bb, es), f16, "o");
      }
      if (st) return st;
      if (kv_raster) {
        st = encode(&prm.k_map[i], raster_spec(*k, *gk, pl(*k), bb, es, ksp), f16, "k");
        if (!st) st = encode(&prm.v_map[i], raster_spec(*v, *gk, pl(*v), bb, es, ksp), f16, "v");
        if (!st && ntxt) st = encode(&prm.kt_map[i], rows_spec(*kt, bsk, pl(*kt), bb, es), f16, "k_txt");
        if (!st && ntxt) st = encode(&prm.vt_map[i], rows_spec(*vt, bsk, pl(*vt), bb, es), f16, "v_txt");
      } else {
        st = encode(&prm.k_map[i], rows_spec(*k, bsk, pl(*k), bb, es), f16, "k");
        if (!st) st = encode(&prm.v_map[i], rows_spec(*v, bsk, pl(*v), bb, es), f16, "v");
      }
      if (st) return st;
    }
    // Tail split of this launch's tiles, when the workspace holds its partials
    // (launches run in stream order, so every launch reuses the workspace).
    const int64_t tiles = nb * H * nq * sub;
    TailPlan tp = tail_plan(tiles, (int64_t)prm.smax * sub);
    const int64_t units = plan_units(tiles, tp);
    if (tp.pieces > 1 && !(workspace && workspace_bytes_avail >= workspace_bytes(units, D) && aligned16(workspace)))
      tp = TailPlan{tiles, 1};
    prm.n_whole = tp.n_whole;
    prm.nsplit = tp.pieces;
    prm.part = tp.pieces > 1 ? static_cast<float*>(workspace) : nullptr;
    prm.part_units = tp.pieces > 1 ? units : 0;
    dim3 grid((unsigned)(tp.n_whole + prm.part_units));
    if (li_status st = launch((int)D, bsk, f16, prm, grid, static_cast<cudaStream_t>(stream))) return st;
    if (tp.pieces > 1) {
      CombineArgs ca;
      memset(&ca, 0, sizeof(ca));
      ca.part = prm.part; ca.part_units = prm.part_units; ca.n_whole = tp.n_whole;
      ca.o = static_cast<uint8_t*>(o->data); ca.o_b = o->stride[0]; ca.o_h = o->stride[1]; ca.o_l = o->stride[2];
      ca.lse = lse; ca.lse_len = nq * bs;
      ca.H = (int)H; ca.b0 = (int)b0; ca.nq = (int)nq; ca.nsplit = tp.pieces; ca.D = (int)D; ca.bs = bs; ca.f16 = f16;
      ca.q_raster = q_raster;
      if (q_raster) {
        ca.T = gq->T; ca.LH = gq->LH; ca.LW = gq->LW; ca.tt = gq->tt; ca.th = gq->th; ca.tw = gq->tw;
        ca.nh = prm.q_nh; ca.nw = prm.q_nw;
      }
      ca.q_len = q->shape[2];
      ca.sub = sub; ca.q_split = prm.q_split; ca.bsk = bsk;
      attn_combine_kernel<<<dim3((unsigned)(tiles - tp.n_whole), (unsigned)(bsk / kCombRows)), kCombThreads, 0,
                            static_cast<cudaStream_t>(stream)>>>(ca);
      if (li_status st = launched("attention combine launch")) return st;
    }
  }
  return LI_OK;
}

}  // namespace attn
}  // namespace li

using namespace li;

extern "C" li_status li_sparse_attn_workspace_bytes(int64_t batch, int64_t heads, int64_t n_q_blocks,
                                                    int64_t max_blocks_per_row, int32_t head_dim, int32_t block_size,
                                                    int64_t* bytes) {
  if (!bytes) return fail(LI_ERR_INVALID_ARG, "bytes is required");
  if (batch < 0 || heads < 0 || n_q_blocks < 0 || max_blocks_per_row < 0) return fail(LI_ERR_SHAPE, "negative shape");
  *bytes = attn::workspace_bytes(attn::call_units(batch, heads, n_q_blocks, max_blocks_per_row, block_size == 256 ? 2 : 1),
                                 head_dim);
  return LI_OK;
}

extern "C" li_status li_sparse_attn_tiled(const li_view4* q, const li_view4* k, const li_view4* v,
                                          const li_index_view* idx, int32_t bs, float sm_scale, li_view4* o,
                                          float* lse, uint32_t* err_word, void* workspace, int64_t workspace_bytes,
                                          void* stream) {
  return attn::run(q, false, nullptr, k, v, false, nullptr, nullptr, nullptr, bs, idx, sm_scale, o, lse, err_word,
                   workspace, workspace_bytes, stream);
}

extern "C" li_status li_sparse_attn_raster(const li_view4* q, li_grid3d grid_q, const li_view4* k_txt,
                                           const li_view4* v_txt, const li_view4* k_vis, const li_view4* v_vis,
                                           li_grid3d grid_k, const li_index_view* idx, float sm_scale, li_view4* o,
                                           float* lse, uint32_t* err_word, void* workspace, int64_t workspace_bytes,
                                           void* stream) {
  if (grid_q.tt != grid_k.tt || grid_q.th != grid_k.th || grid_q.tw != grid_k.tw || grid_q.LH != grid_k.LH ||
      grid_q.LW != grid_k.LW)
    return fail(LI_ERR_SHAPE, "grid_q and grid_k must share the latent size and tile");
  const int bs = grid_q.tt * grid_q.th * grid_q.tw;
  return attn::run(q, true, &grid_q, k_vis, v_vis, true, &grid_k, k_txt, v_txt, bs, idx, sm_scale, o, lse, err_word,
                   workspace, workspace_bytes, stream);
}
