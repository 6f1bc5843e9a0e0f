// All-to-all over NVLink peer memory for the head-sharded stack (the Ulysses
// sequence<->head re-layout around the sparse attention).
//
// Every rank pushes: chunk p of its send buffer (rows of `row_bytes`) is
// written with 16-byte stores straight into rank p's receive buffer, at a
// per-source offset and row stride chosen by the caller (so the output side
// lands directly in the [s, H, D] layout the O projection reads). A row may be
// split: its first `split_bytes` go to the receive buffer and the rest to a
// second buffer of rank p (the stack sends each token's q there and its k, v
// straight into the rank's resident K/V buffer). No NCCL, no copy engine, no
// multicast: plain st.global to peer addresses opened through CUDA IPC.
//
// Completion: each CTA fences its stores at system scope and takes a ticket;
// the last CTA raises flag[rank] = epoch on every peer, then waits (bounded by
// %globaltimer) until every peer has raised its flag here. The kernel therefore
// ends only when this rank's receive buffer is complete. On timeout it sets
// LI_DEVERR_TIMEOUT in the error word and returns.
//
// Reuse: the caller alternates two receive buffers by call parity. A peer can
// start writing call e+2 into the buffer of call e only after this rank has
// joined call e+1, which its stream issues after everything that reads call e's
// buffer.
#include <cstring>

#include "li_common.cuh"

namespace li {
namespace {

constexpr int kA2AThreads = 256;
constexpr uint64_t kA2ATimeoutNs = 2000000000ull;

struct A2AArgs {
  const uint8_t* src;
  int64_t src_chunk_stride, src_row_stride;  // bytes
  uint8_t* dst[LI_A2A_MAX_RANKS];            // receive-buffer base of every rank
  int64_t dst_offset, dst_row_stride;        // bytes, on every destination
  uint8_t* dst2[LI_A2A_MAX_RANKS];           // second destination of every rank (split rows)
  int64_t dst2_offset, dst2_row_stride;      // bytes
  int64_t split_vecs;                        // 16-byte vectors of a row that go to dst (all: no split)
  int64_t rows, row_bytes;
  uint32_t* flags[LI_A2A_MAX_RANKS];         // flag array of every rank (slot = source rank)
  uint32_t* my_flags;
  uint32_t* counter;
  uint32_t* err;
  uint32_t* epoch_word;  // optional: epoch = *epoch_word + 1, stored back at the end
  uint32_t epoch;
  int32_t world, rank;
};

__device__ __forceinline__ uint64_t a2a_timer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kA2AThreads) a2a_push_kernel(const A2AArgs a) {
  const int64_t v_per_row = a.row_bytes / 16;
  const int64_t v_per_chunk = a.rows * v_per_row;
  // CTAs are dealt round-robin over the destinations, starting with the rank
  // after this one: every rank writes to all of its peers at once and every rank
  // receives from all of them at once. (Walking the chunks in order would send
  // every rank's traffic to the same destination at the same time.)
  const int W = a.world;
  const int slot = (int)(blockIdx.x % W);
  const int p = (a.rank + 1 + slot) % W;
  const int64_t n_cta = (gridDim.x - slot + W - 1) / W;  // CTAs serving this destination
  const uint8_t* src = a.src + p * a.src_chunk_stride;
  uint8_t* dst = a.dst[p] + a.dst_offset;
  uint8_t* dst2 = a.split_vecs < v_per_row ? a.dst2[p] + a.dst2_offset : nullptr;
  for (int64_t i = (int64_t)(blockIdx.x / W) * kA2AThreads + threadIdx.x; i < v_per_chunk;
       i += n_cta * kA2AThreads) {
    const int64_t r = i / v_per_row, c = i % v_per_row;
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + r * a.src_row_stride) + c);
    if (c < a.split_vecs) *(reinterpret_cast<uint4*>(dst + r * a.dst_row_stride) + c) = v;
    else *(reinterpret_cast<uint4*>(dst2 + r * a.dst2_row_stride) + (c - a.split_vecs)) = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x != 0) return;
  const uint32_t ticket = atomicAdd(a.counter, 1u);
  if (ticket != gridDim.x - 1) return;
  // Last CTA: every CTA's stores are fenced. Publish, then wait for the peers.
  // Only this CTA uses the epoch, so a device-held epoch is read here (the
  // previous call on this stream stored it before this launch began).
  const uint32_t epoch = a.epoch_word ? *(volatile uint32_t*)a.epoch_word + 1u : a.epoch;
  __threadfence_system();
  for (int p = 0; p < a.world; ++p) st_release_sys(a.flags[p] + a.rank, epoch);
  const uint64_t t0 = a2a_timer();
  bool timed_out = false;
  for (int p = 0; p < a.world && !timed_out; ++p) {
    uint32_t it = 0;
    // A peer that already finished this call may have raised the next epoch:
    // accept any flag at or past this one (wrap-around compare).
    while ((int32_t)(ld_acquire_sys(a.my_flags + p) - epoch) < 0) {
      if ((++it & 63u) == 0 && a2a_timer() - t0 > kA2ATimeoutNs) {
        if (a.err) atomicOr(a.err, (unsigned)LI_DEVERR_TIMEOUT);
        timed_out = true;
        break;
      }
    }
  }
  // The epoch advances on timeout too, so later calls stay numbered like the peers'.
  if (a.epoch_word) *a.epoch_word = epoch;
  *a.counter = 0u;  // ready for the next call on this stream
}

}  // namespace
}  // namespace li

using namespace li;

extern "C" li_status li_ipc_alloc(int64_t bytes, void** ptr, void* handle_out) {
  if (!ptr || !handle_out || bytes <= 0) return fail(LI_ERR_INVALID_ARG, "bytes, ptr and handle_out are required");
  void* p = nullptr;
  if (li_status st = cuda_status(cudaMalloc(&p, (size_t)bytes), "cudaMalloc (exchange buffer)")) return st;
  if (li_status st = cuda_status(cudaMemset(p, 0, (size_t)bytes), "cudaMemset (exchange buffer)")) {
    cudaFree(p);
    return st;
  }
  cudaIpcMemHandle_t h;
  if (li_status st = cuda_status(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle")) {
    cudaFree(p);
    return st;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == LI_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return LI_OK;
}

extern "C" li_status li_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(LI_ERR_INVALID_ARG, "handle and ptr are required");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

extern "C" li_status li_ipc_close(void* ptr) {
  if (!ptr) return LI_OK;
  return cuda_status(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
}

extern "C" li_status li_ipc_free(void* ptr) {
  if (!ptr) return LI_OK;
  return cuda_status(cudaFree(ptr), "cudaFree (exchange buffer)");
}

extern "C" li_status li_a2a_push(const li_a2a_desc* d, void* stream) {
  if (!d || !d->src || !d->my_flags || !d->counter) return fail(LI_ERR_INVALID_ARG, "descriptor incomplete");
  if (d->world < 1 || d->world > LI_A2A_MAX_RANKS || d->rank < 0 || d->rank >= d->world)
    return fail(LI_ERR_INVALID_ARG, "rank %d of world %d", d->rank, d->world);
  if (d->rows <= 0 || d->row_bytes <= 0 || d->row_bytes % 16)
    return fail(LI_ERR_SHAPE, "rows and row_bytes (multiple of 16) must be positive");
  if (!aligned16(d->src) || d->src_chunk_stride % 16 || d->src_row_stride % 16 || d->dst_offset % 16 ||
      d->dst_row_stride % 16)
    return fail(LI_ERR_ALIGNMENT, "exchange pointers, offsets and strides must be 16-byte multiples");
  const bool split = d->split_bytes != 0;
  if (split && (d->split_bytes < 16 || d->split_bytes >= d->row_bytes || d->split_bytes % 16 ||
                d->dst2_offset % 16 || d->dst2_row_stride % 16 || d->dst2_offset < 0 || d->dst2_row_stride < 0))
    return fail(LI_ERR_ALIGNMENT, "split_bytes must be a 16-byte multiple inside the row, and dst2 offsets 16-byte "
                                  "multiples");
  if (d->dst_offset < 0 || d->dst_row_stride < 0) return fail(LI_ERR_INVALID_ARG, "negative offset or stride");
  const int64_t first = split ? d->split_bytes : d->row_bytes;
  const int64_t dst_extent = d->dst_offset + (d->rows - 1) * d->dst_row_stride + first;
  if (dst_extent > d->dst_bytes) return fail(LI_ERR_OUT_OF_BOUNDS, "exchange writes past the receive buffer");
  if (split && d->dst2_offset + (d->rows - 1) * d->dst2_row_stride + (d->row_bytes - first) > d->dst2_bytes)
    return fail(LI_ERR_OUT_OF_BOUNDS, "exchange writes past the second destination");
  A2AArgs a;
  memset(&a, 0, sizeof(a));
  a.src = static_cast<const uint8_t*>(d->src);
  a.src_chunk_stride = d->src_chunk_stride; a.src_row_stride = d->src_row_stride;
  for (int p = 0; p < d->world; ++p) {
    if (!d->dst[p] || !d->flags[p] || !aligned16(d->dst[p]))
      return fail(LI_ERR_INVALID_ARG, "rank %d: receive buffer or flag array missing or unaligned", p);
    a.dst[p] = static_cast<uint8_t*>(d->dst[p]);
    a.flags[p] = d->flags[p];
    if (split) {
      if (!d->dst2[p] || !aligned16(d->dst2[p]))
        return fail(LI_ERR_INVALID_ARG, "rank %d: second destination missing or unaligned", p);
      a.dst2[p] = static_cast<uint8_t*>(d->dst2[p]);
    }
  }
  a.dst_offset = d->dst_offset; a.dst_row_stride = d->dst_row_stride;
  a.dst2_offset = d->dst2_offset; a.dst2_row_stride = d->dst2_row_stride;
  a.split_vecs = first / 16;
  a.rows = d->rows; a.row_bytes = d->row_bytes;
  a.my_flags = d->my_flags; a.counter = d->counter; a.err = d->err_word; a.epoch_word = d->epoch_word;
  a.epoch = d->epoch; a.world = d->world; a.rank = d->rank;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // A multiple of world CTAs, at least one per destination, about four vectors
  // per thread, at most four CTAs per SM.
  const int64_t vecs = (int64_t)d->world * d->rows * (d->row_bytes / 16);
  const int64_t want = std::min<int64_t>(ceil_div(vecs, (int64_t)kA2AThreads * 4), (int64_t)sms * 4);
  const unsigned grid = (unsigned)(std::max<int64_t>(1, want / d->world) * d->world);
  a2a_push_kernel<<<grid, kA2AThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launched("a2a_push_kernel launch");
}
