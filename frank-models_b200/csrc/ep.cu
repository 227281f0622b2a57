// Expert-parallel exchange over NVLink peer memory.
//
// The experts of the MoE block are split evenly over P ranks (El = E / P
// each, contiguous).  Every rank's expert-sorted slots are therefore grouped
// by destination rank already.  Given the all-gathered per-expert counts
// C[q][g] (rows rank q routes to global expert g), these kernels
//   - plan:     where each of my (destination rank, expert) chunks lands in
//               the destination's expert-major receive buffer, and my own
//               experts' row offsets;                       (ep_plan_kernel)
//   - dispatch: gather my token rows and their gate weights and store them
//               straight into the destination ranks' receive buffers
//               (P2P stores over NVLink; no staging copy)   (ep_dispatch_kernel)
//   - return map: for every row of my receive buffer, the source rank and
//               the row of that rank's expert-sorted order it belongs to,
//               so the down-GEMM epilogue can store its result directly into
//               the source rank's return buffer             (ep_return_map_kernel)
// Nothing here waits on another GPU: ordering between ranks is established
// by the caller with stream-ordered collectives (NCCL) between the steps.
#include "common.cuh"

namespace {

constexpr int kMaxPeers = 8;

struct PeerRows {
  void* x[kMaxPeers];   // receive buffers [capacity, H] of every rank
  float* w[kMaxPeers];  // receive gate weights [capacity] of every rank
};

// C: [P][E] int32 (all ranks' per-expert counts).  One block.
//   dst_base[g]  (g = p*El + e): first row of my chunk for expert g in rank
//                p's expert-major buffer = sum_{e'<e} sum_q C[q][p*El+e']
//                + sum_{q<me} C[q][g]
//   local_off[e] (e = 0..El): sum_{e'<e} sum_q C[q][me*El+e']
__global__ void ep_plan_kernel(const int32_t* __restrict__ C, int P, int El, int me, int32_t* __restrict__ dst_base,
                               int32_t* __restrict__ local_off, int64_t capacity, int32_t* __restrict__ err) {
  const int E = P * El;
  // a negative entry is not a count: then nothing is placed or computed
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < P * E; i += blockDim.x)
    if (C[i] < 0) s_bad = 1;
  __syncthreads();
  if (s_bad) {
    if (threadIdx.x == 0) atomicExch(err, FRANK_EINVAL);
    for (int g = threadIdx.x; g < E; g += blockDim.x) dst_base[g] = (int32_t)capacity;  // refused by the dispatch
    for (int e = threadIdx.x; e <= El; e += blockDim.x) local_off[e] = 0;              // no rows for the GEMMs
    return;
  }
  for (int g = threadIdx.x; g < E; g += blockDim.x) {
    const int p = g / El, e = g - p * El;
    int32_t base = 0;
    for (int e2 = 0; e2 < e; ++e2)
      for (int q = 0; q < P; ++q) base += C[q * E + p * El + e2];
    for (int q = 0; q < me; ++q) base += C[q * E + g];
    dst_base[g] = base;
  }
  for (int e = threadIdx.x; e <= El; e += blockDim.x) {
    int32_t off = 0;
    for (int e2 = 0; e2 < e; ++e2)
      for (int q = 0; q < P; ++q) off += C[q * E + me * El + e2];
    // rows past the receive buffer were never stored there: the GEMMs must
    // not read them (nor map them back), so the offsets stop at capacity
    if ((int64_t)off > capacity) {
      off = (int32_t)capacity;
      atomicExch(err, FRANK_EINVAL);
    }
    local_off[e] = off;
  }
}

// Block (q, e) fills the rows my receive buffer holds from rank q for my
// local expert e: row_rank = q, row_pos = position in q's expert-sorted order.
__global__ void ep_return_map_kernel(const int32_t* __restrict__ C, int P, int El, int me,
                                     const int32_t* __restrict__ local_off, int32_t* __restrict__ row_rank,
                                     int32_t* __restrict__ row_pos, int64_t capacity) {
  const int E = P * El;
  const int q = blockIdx.x / El, e = blockIdx.x - (blockIdx.x / El) * El;
  const int g = me * El + e;
  __shared__ int32_t s_start, s_src, s_len;
  if (threadIdx.x == 0) {
    int32_t start = local_off[e];
    for (int q2 = 0; q2 < q; ++q2) start += C[q2 * E + g];
    int32_t src = 0;
    for (int g2 = 0; g2 < g; ++g2) src += C[q * E + g2];
    s_start = start;
    s_src = src;
    s_len = C[q * E + g];
  }
  __syncthreads();
  if (s_start < 0 || s_len < 0) return;  // counts are never negative; refused by ep_plan_kernel
  for (int i = threadIdx.x; i < s_len && (int64_t)s_start + i < capacity; i += blockDim.x) {
    row_rank[s_start + i] = q;
    row_pos[s_start + i] = s_src + i;
  }
}

// One warp per expert-sorted slot r of this rank: destination rank p and
// row from the plan, the token row gathered from x, stored with 16-byte
// vectors into rank p's receive buffer (a peer address when p != me).
__global__ void ep_dispatch_kernel(const uint4* __restrict__ x, int64_t T, int64_t vec_per_row,
                                   const float* __restrict__ w, const int32_t* __restrict__ sorted_slots,
                                   const int32_t* __restrict__ offsets, int E, int El, int64_t n,
                                   const int32_t* __restrict__ dst_base, int64_t capacity, int32_t* __restrict__ err,
                                   PeerRows peers) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); r < n;
       r += (int64_t)gridDim.x * (blockDim.x / 32)) {
    int lo = 0, hi = E;  // expert g: offsets[g] <= r < offsets[g+1]
    while (hi - lo > 1) {
      int mid = (lo + hi) >> 1;
      if (offsets[mid] <= r) lo = mid; else hi = mid;
    }
    const int g = lo, p = g / El;
    const int64_t dst = (int64_t)dst_base[g] + (r - offsets[g]);
    if (dst < 0 || dst >= capacity) {  // never stores outside the peer's buffer
      if (lane == 0) atomicExch(err, FRANK_EINVAL);
      continue;
    }
    const int32_t s = sorted_slots[r];
    const uint4* src = x + (int64_t)(s % T) * vec_per_row;
    uint4* d = reinterpret_cast<uint4*>(peers.x[p]) + dst * vec_per_row;
    // all loads of a 16-vector round in flight before the (remote) stores
    for (int64_t v0 = 0; v0 < vec_per_row; v0 += 32 * 16) {
      uint4 buf[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int64_t v = v0 + lane + 32 * i;
        if (v < vec_per_row) buf[i] = __ldg(src + v);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int64_t v = v0 + lane + 32 * i;
        if (v < vec_per_row) d[v] = buf[i];
      }
    }
    if (lane == 0) peers.w[p][dst] = w[s];
  }
  __threadfence_system();
}

}  // namespace

extern "C" {

int frank_ep_plan(const int32_t* counts_all, int P, int El, int rank, int32_t* dst_base, int32_t* local_offsets,
                  int32_t* row_rank, int32_t* row_pos, int64_t capacity, int32_t* overflow, void* stream) {
  if (P < 1 || P > kMaxPeers || El < 1 || rank < 0 || rank >= P || P * El > 1024) {
    frank::set_error("ep_plan: P=%d El=%d rank=%d out of range (P <= %d, P*El <= 1024)", P, El, rank, kMaxPeers);
    return FRANK_EINVAL;
  }
  cudaStream_t st = frank::as_stream(stream);
  ep_plan_kernel<<<1, 1024, 0, st>>>(counts_all, P, El, rank, dst_base, local_offsets, capacity,
                                     overflow ? overflow : frank::device_error_word());
  FRANK_LAUNCH_CHECK();
  ep_return_map_kernel<<<P * El, 256, 0, st>>>(counts_all, P, El, rank, local_offsets, row_rank, row_pos,
                                                  capacity);
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

int frank_ep_dispatch(const void* x, int64_t T, int64_t H, const float* w, const int32_t* sorted_slots,
                      const int32_t* offsets, int64_t E, int64_t El, int64_t n_slots, const int32_t* dst_base,
                      void* const* peer_x, float* const* peer_w, int P, int64_t capacity, int32_t* overflow,
                      void* stream) {
  if (P < 1 || P > kMaxPeers || El < 1 || E != El * P) {
    frank::set_error("ep_dispatch: P=%d El=%lld E=%lld inconsistent", P, (long long)El, (long long)E);
    return FRANK_EINVAL;
  }
  if ((H * 2) % 16 != 0 || (uintptr_t)x % 16 != 0) {
    frank::set_error("ep_dispatch: bf16 rows must be 16-byte multiples and aligned (H=%lld)", (long long)H);
    return FRANK_EINVAL;
  }
  if (n_slots == 0) return FRANK_OK;
  PeerRows peers;
  for (int i = 0; i < kMaxPeers; ++i) {
    peers.x[i] = i < P ? peer_x[i] : nullptr;
    peers.w[i] = i < P ? peer_w[i] : nullptr;
    if (i < P && (((uintptr_t)peers.x[i] % 16) != 0 || !peers.w[i])) {
      frank::set_error("ep_dispatch: peer buffer %d missing or misaligned", i);
      return FRANK_EINVAL;
    }
  }
  int64_t blocks = (n_slots + 7) / 8;
  const int64_t cap = (int64_t)frank::num_sms() * 8;
  ep_dispatch_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, frank::as_stream(stream)>>>(
      (const uint4*)x, T, H * 2 / 16, w, sorted_slots, offsets, (int)E, (int)El, n_slots, dst_base, capacity,
      overflow ? overflow : frank::device_error_word(), peers);
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

}  // extern "C"
