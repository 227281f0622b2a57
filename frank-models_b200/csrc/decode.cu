// Decode-sized MoE FFN block (k * T <= E token slots): weight streaming on
// CUDA cores.
//
// With a few tokens an expert receives a handful of rows, so the block is
// bound by reading the active experts' weights from HBM (3 x H x F bf16 per
// active expert) -- tensor cores would idle on 128-row tiles.  Phases:
//   route    router logits; an item is (expert, 8 tokens) and, with fewer
//            items than warps, the warps of a block split H for an item
//            (moe_ffn_block.mlir:54-70);
//   top-k    softmax + top-k + renorm of every token (moe_ffn_block.mlir:
//            72-128), the stable expert permutation and the list of active
//            experts (mul_mat_id.mlir:51-53);
//   gate/up  persistent blocks over (active expert, fr rows of F): the gate
//            and up rows streamed once into shared memory with bulk copies
//            and dotted with the expert's token rows (gathered straight
//            from x), h = gate * silu(up) (swiglu.mlir:37-47);
//   down     persistent blocks over (active expert, hr rows of H):
//            d = down(h) * gate weight, fp32;
//   combine  y[t] = sum of the k slots of t in slot order
//            (moe_ffn_block.mlir:179-206), deterministic.
// decode_fused_kernel runs all phases in one cooperative launch with three
// grid barriers (after route, gate/up and down): every block computes the
// top-k and the permutation of all tokens itself.  Blocks have eight compute
// warps plus one warp that issues the streaming phases' bulk copies.  FRANK_DECODE_FUSED=0 runs
// the same bodies as five launches chained by programmatic dependent launch.
// No atomics on data: results are deterministic and identical in both forms.
#include <cstdlib>

#include "common.cuh"
#include "mbarrier.cuh"
#include "topk.cuh"

namespace {

using namespace frank_topk;

constexpr int kThreads = 256;           // compute threads (warps 0 .. kWarps-1)
constexpr int kWarps = kThreads / 32;
constexpr int kBlockThreads = kThreads + 32;  // + the streaming phases' bulk-copy producer warp
constexpr int kRouteTok = 8;    // tokens per route warp item
constexpr int kMaxSlots = kMaxE; // k * T handled by the decode path (k * T <= E)
constexpr int kRC = 8;          // token rows per pass over an expert's weights

__device__ __forceinline__ void bf16x8_to_f32(uint4 u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

template <class TW>
__device__ __forceinline__ void load8_w(const TW* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8_w<float>(const float* p, float (&v)[8]) {
  float4 a = __ldg(reinterpret_cast<const float4*>(p));
  float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8_w<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(p)), v);
}

struct DecodeWs {
  float* logits;        // [E, T]
  float* w;             // [k, T] gate weights
  int32_t* ids;         // [k, T]
  int32_t* sorted_slots;
  int32_t* offsets;     // [E + 1]
  int32_t* slot_pos;
  float* wsorted;
  __nv_bfloat16* hs;    // [k*T, F]
  int32_t* active;      // experts with at least one row, ascending
  int32_t* nactive;
  float* d;             // [k*T, H] down output x gate weight
  int32_t* err;         // device error word (bounded waits)
  unsigned* gbar;       // grid-barrier counter of the fused kernel (zeroed per call)
  const float* res;     // optional fp32 [T, H] residual added to y (may alias y)
  int n_slots;          // k * T
};

// Routing tables of one call in shared memory: expert row offsets [E+1],
// active experts [E] (first *nact valid), token of each expert-sorted row,
// gate weight of each expert-sorted row.
struct Meta {
  int32_t* off;
  int32_t* act;
  int32_t* nact;
  int32_t* tok;
  float* w;
};

// Programmatic dependent launch: a kernel's blocks may start while the
// previous kernel of the stream finishes; they wait here for its results.
__device__ __forceinline__ void wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_next_grid() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Barrier of the kThreads compute threads (warps 0 .. kWarps-1): the
// routing phases run without the producer warp.
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }

// ----------------------------------------------------------------- route --
// logits[e, t] = Wr[e] . x[t] for items (expert e, kRouteTok tokens).  When
// there are fewer items than warps in the grid, wpi warps of one block split
// H for each item (one dependent HBM round trip per warp instead of H/256)
// and the block sums their partials in shared memory.  red: [kWarps][kRouteTok].
template <class TW>
__device__ __forceinline__ void route_body(const __nv_bfloat16* __restrict__ x, const TW* __restrict__ wr, int T,
                                           int H, int E, const DecodeWs& ws, float* red, int bid, int nblk) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tchunks = (T + kRouteTok - 1) / kRouteTok;
  const int items = E * tchunks;
  int wpi = kWarps;
  while (wpi > 1 && (int64_t)items * wpi > (int64_t)nblk * kWarps) wpi >>= 1;
  const int ipb = kWarps / wpi;  // items per block per round
  const int sub = warp % wpi, slot = warp / wpi;
  for (int base = bid * ipb; base < items; base += nblk * ipb) {  // uniform across the block
    const int item = base + slot;
    float acc[kRouteTok];
#pragma unroll
    for (int a = 0; a < kRouteTok; ++a) acc[a] = 0.f;
    int e = 0, t0 = 0;
    if (item < items) {
      e = item / tchunks;
      t0 = (item - e * tchunks) * kRouteTok;
#pragma unroll 4
      for (int h = (sub * 32 + lane) * 8; h < H; h += wpi * 256) {
        float wv[8];
        load8_w(wr + (int64_t)e * H + h, wv);
#pragma unroll
        for (int a = 0; a < kRouteTok; ++a) {
          if (t0 + a < T) {
            float xv[8];
            bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(x + (int64_t)(t0 + a) * H + h)), xv);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[a] = fmaf(wv[i], xv[i], acc[a]);
          }
        }
      }
    }
#pragma unroll
    for (int a = 0; a < kRouteTok; ++a) {
      float v = acc[a];
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[warp * kRouteTok + a] = v;
    }
    consumer_sync();
    if (sub == 0 && lane < kRouteTok && item < items && t0 + lane < T) {
      float v = 0.f;
      for (int s2 = 0; s2 < wpi; ++s2) v += red[(slot * wpi + s2) * kRouteTok + lane];
      ws.logits[(int64_t)e * T + t0 + lane] = v;
    }
    consumer_sync();
  }
}


template <class TW>
__global__ void __launch_bounds__(kThreads)
decode_route_kernel(const __nv_bfloat16* __restrict__ x, const TW* __restrict__ wr, int T, int H, int E, int k,
                    int normalize, DecodeWs ws) {
  __shared__ float red[kWarps * kRouteTok];
  allow_next_grid();
  route_body<TW>(x, wr, T, H, E, ws, red, blockIdx.x, gridDim.x);
}

// One block: softmax + top-k + renorm for every token, the stable expert
// permutation (same order as argsort(ids.reshape(-1), stable)) and the list of
// active experts.
// Shared scratch of finalize_body: lg [kWarps][kMaxE] f32, running [kMaxE+1],
// warp_cnt [kWarps][kMaxE], rank [kMaxSlots] (int32).
constexpr size_t kFinalizeSmem = sizeof(float) * kWarps * kMaxE + sizeof(int32_t) * (kMaxE + 1 + kWarps * kMaxE + kMaxSlots);

// Descending top-k (ties to the lower expert index) of one token's
// probabilities p[E] by one warp, renormalised when asked: the selection
// steps of warp_softmax_topk.
__device__ __forceinline__ void warp_softmax_topk_probs(const float* p_in, int E, int k, int normalize, float* w_out,
                                                        int32_t* id_out, int T, int t) {
  const int lane = threadIdx.x & 31;
  constexpr int kPer = kMaxE / 32;
  float p[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? p_in[e] : -1.f;  // probabilities are >= 0; -1 marks "absent"
  }
  float wsum = 0.f;
  for (int j = 0; j < k; ++j) {
    float bv = -2.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (p[i] > bv) { bv = p[i]; bi = lane + 32 * i; }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (lane + 32 * i == bi) p[i] = -2.f;
    wsum += bv;  // ascending j, as numpy's sum over a short axis
    if (lane == 0) {
      id_out[j * T + t] = bi;
      w_out[j * T + t] = bv;
    }
  }
  __syncwarp();
  if (normalize && lane == 0)
    for (int j = 0; j < k; ++j) w_out[j * T + t] = w_out[j * T + t] / wsum;
  __syncwarp();
}

// Softmax over the E experts and the descending top-k (ties to the lower
// expert index), renormalised when asked, of all T tokens by one block.
// Warps compute the probabilities (one token per warp, the arithmetic of
// warp_softmax_topk).  With at most one (token, expert) pair per thread,
// every thread ranks its pair by counting the larger probabilities of its
// token (no serial k-step selection); otherwise one warp selects per token.
// Both give the same ids and weights.  prob: shared [T][E]; w_out / id_out:
// [k, T], shared or global.
__device__ __forceinline__ void block_softmax_topk(const float* logits, int T, int E, int k, int normalize,
                                                   float* prob, float* w_out, int32_t* id_out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kPer = kMaxE / 32;
  for (int t = warp; t < T; t += kWarps) {
    float v[kPer];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? __ldcg(logits + (int64_t)e * T + t) : -INFINITY;
      mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? expf(v[i] - mx) : 0.f;
      sum += v[i];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      if (e < E) prob[t * E + e] = v[i] / sum;
    }
  }
  consumer_sync();
  if (T * E > kThreads) {
    // more pairs than threads: a serial k-step selection per token and warp
    for (int t = warp; t < T; t += kWarps) warp_softmax_topk_probs(prob + t * E, E, k, normalize, w_out, id_out, T, t);
    consumer_sync();
    return;
  }
  for (int idx = threadIdx.x; idx < T * E; idx += kThreads) {
    const int t = idx / E, e = idx - t * E;
    const float* pt = prob + t * E;
    const float p = pt[e];
    int r = 0;
#pragma unroll 4
    for (int u = 0; u < E; ++u) {
      const float q = pt[u];
      r += (q > p) | ((q == p) & (u < e));
    }
    if (r < k) {
      id_out[r * T + t] = e;
      w_out[r * T + t] = p;
    }
  }
  consumer_sync();
  if (normalize) {
    for (int t = threadIdx.x; t < T; t += kThreads) {
      float s = 0.f;
      for (int j = 0; j < k; ++j) s += w_out[j * T + t];  // ascending j, as numpy's sum over a short axis
      for (int j = 0; j < k; ++j) w_out[j * T + t] = w_out[j * T + t] / s;
    }
    consumer_sync();
  }
}

// One block: the stable permutation of the top-k slots ids / gate weights wts
// ([k, T], written earlier by this block) and the active list, into the
// block's shared tables m; the writer block also stores them (and slot_pos)
// to global memory.
__device__ __forceinline__ void permute_body(int T, int E, int k, const DecodeWs& ws, uint8_t* scratch, Meta m,
                                             const int32_t* ids, const float* wts, bool writer) {
  float* lg = reinterpret_cast<float*>(scratch);
  int32_t* running = reinterpret_cast<int32_t*>(lg + kWarps * kMaxE);
  int32_t* warp_cnt = running + kMaxE + 1;
  int32_t* rank = warp_cnt + kWarps * kMaxE;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // stable counting sort of the n = k*T flat slots by expert (same order as
  // argsort(ids.reshape(-1), stable)); one block, warp-level ranks
  const int n = k * T;
  for (int e = threadIdx.x; e < E; e += kThreads) {
    running[e] = 0;
    for (int w2 = 0; w2 < kWarps; ++w2) warp_cnt[w2 * kMaxE + e] = 0;
  }
  consumer_sync();
  for (int base = 0; base < n; base += kThreads) {
    const int s = base + threadIdx.x;
    const int e = s < n ? ids[s] : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_w = __popc(peers & ((1u << lane) - 1u));
    const int leader = __ffs(peers) - 1;
    if (e >= 0 && lane == leader) warp_cnt[warp * kMaxE + e] = __popc(peers);
    consumer_sync();
    int pos = 0;
    bool last = false;
    if (e >= 0) {
      int before = 0;
      for (int w2 = 0; w2 < warp; ++w2) before += warp_cnt[w2 * kMaxE + e];
      pos = running[e] + before + rank_w;
      rank[s] = pos;
      last = (lane == 31 - __clz(peers));
      for (int w2 = warp + 1; w2 < kWarps && last; ++w2)
        if (warp_cnt[w2 * kMaxE + e] != 0) last = false;
    }
    consumer_sync();
    if (last) running[e] = pos + 1;
    if (e >= 0 && lane == leader) warp_cnt[warp * kMaxE + e] = 0;
    consumer_sync();
  }
  if (warp == 0) {  // exclusive scan of the counts and the active-expert list (E <= 256)
    int carry = 0, na = 0;
    for (int base = 0; base < E; base += 32) {
      const int e = base + lane;
      const int c = e < E ? running[e] : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      if (e < E) {
        m.off[e] = carry + incl - c;
        running[e] = carry + incl - c;
        if (writer) ws.offsets[e] = carry + incl - c;
      }
      const unsigned act = __ballot_sync(0xffffffffu, c > 0);
      if (c > 0) {
        const int slot = na + __popc(act & ((1u << lane) - 1u));
        m.act[slot] = e;
        if (writer) ws.active[slot] = e;
      }
      na += __popc(act);
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      m.off[E] = carry;
      *m.nact = na;
      if (writer) {
        ws.offsets[E] = carry;
        *ws.nactive = na;
      }
    }
  }
  consumer_sync();
  for (int s = threadIdx.x; s < n; s += kThreads) {
    const int32_t pos = running[ids[s]] + rank[s];
    const float w = wts[s];
    m.tok[pos] = s % T;
    m.w[pos] = w;
    if (writer) {
      ws.sorted_slots[pos] = s;
      ws.slot_pos[s] = pos;
      ws.wsorted[pos] = w;
    }
  }
  consumer_sync();
}

// permute_body for at most 32 slots (k * T <= 32): the same tables from one
// barrier.  Every compute thread counts the slots below its experts for the
// offsets; warp 0 ranks each slot by shuffles (stable: expert, then slot)
// and lists the active experts in ascending order.
__device__ __forceinline__ void small_permute_body(int T, int E, int k, const DecodeWs& ws, Meta m,
                                                   const int32_t* ids, const float* wts, bool writer) {
  const int n = k * T;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e <= E; e += kThreads) {
    int c = 0;
    for (int s2 = 0; s2 < n; ++s2) c += ids[s2] < e;
    m.off[e] = c;
    if (writer) ws.offsets[e] = c;
  }
  if (warp == 0) {
    const int e = lane < n ? ids[lane] : 0x7fffffff;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const bool first = lane < n && (peers & ((1u << lane) - 1u)) == 0u;  // first slot of its expert
    const unsigned firsts = __ballot_sync(0xffffffffu, first);
    int pos = 0, aidx = 0;
    for (int t = 0; t < n; ++t) {
      const int et = __shfl_sync(0xffffffffu, e, t);
      pos += (et < e) | ((et == e) & (t < lane));
      aidx += (int)((firsts >> t) & 1u) & (et < e);
    }
    if (first) {
      m.act[aidx] = e;
      if (writer) ws.active[aidx] = e;
    }
    if (lane == 0) {
      *m.nact = __popc(firsts);
      if (writer) *ws.nactive = __popc(firsts);
    }
    if (lane < n) {
      const float w = wts[lane];
      m.tok[pos] = lane % T;
      m.w[pos] = w;
      if (writer) {
        ws.sorted_slots[pos] = lane;
        ws.slot_pos[lane] = pos;
        ws.wsorted[pos] = w;
      }
    }
  }
  consumer_sync();
}

__device__ __forceinline__ void finalize_body(int T, int E, int k, int normalize, const DecodeWs& ws, uint8_t* scratch,
                                              float* prob, Meta m) {
  block_softmax_topk(ws.logits, T, E, k, normalize, prob, ws.w, ws.ids);
  permute_body(T, E, k, ws, scratch, m, ws.ids, ws.w, true);
}


__global__ void __launch_bounds__(kThreads)
decode_finalize_kernel(int T, int E, int k, int normalize, DecodeWs ws) {
  __shared__ __align__(16) uint8_t scratch[kFinalizeSmem];
  extern __shared__ __align__(16) float prob[];  // [T][E] (dynamic)
  __shared__ int32_t m_off[kMaxE + 1], m_act[kMaxE], m_nact, m_tok[kMaxSlots];
  __shared__ float m_w[kMaxSlots];
  wait_prior_grid();
  allow_next_grid();
  finalize_body(T, E, k, normalize, ws, scratch, prob, Meta{m_off, m_act, &m_nact, m_tok, m_w});
}


__device__ __forceinline__ Meta load_meta(const DecodeWs& ws, int T, int E, int32_t* off, int32_t* act, int32_t* nact,
                                          int32_t* tok, float* w) {
  for (int i = threadIdx.x; i <= E; i += blockDim.x) off[i] = __ldcg(ws.offsets + i);
  for (int i = threadIdx.x; i < E; i += blockDim.x) act[i] = __ldcg(ws.active + i);
  for (int i = threadIdx.x; i < ws.n_slots; i += blockDim.x) {
    tok[i] = __ldcg(ws.sorted_slots + i) % T;
    w[i] = __ldcg(ws.wsorted + i);
  }
  if (threadIdx.x == 0) *nact = __ldcg(ws.nactive);
  __syncthreads();
  return Meta{off, act, nact, tok, w};
}

// ----------------------------------------------- weight-streaming GEMVs --
// Both GEMV kernels stream contiguous chunks of an expert's weight rows from
// HBM into a ring of shared-memory stages with 1-D bulk copies
// (cp.async.bulk, one mbarrier per stage), so that every SM keeps 100+ KB of
// weights in flight; the token rows of the chunk's expert are staged next to
// them and every warp dots whole rows out of shared memory.  Items are
// (active expert, chunk of rows), spread over persistent blocks.
using namespace frank_mbar;

// gate/up: item = (active expert e, fr rows of F starting at f0): stage =
// fr gate rows then fr up rows ([2][fr][H] bf16).  Warp w < fr computes row
// f0 + w for each token row: h = gate . x * silu(up . x).
__device__ __forceinline__ void gateup_body(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w_gate,
                     const __nv_bfloat16* __restrict__ w_up, int T, int H, int F, int E, int fr, int rcap, int stages,
                     DecodeWs ws, int bid, int nblk, uint8_t* dsm_raw, uint64_t* full, uint64_t* empty,
                     int* s_abort, Meta m) {
  // routing tables in shared memory: refilling a stage needs no global round trip
  const int32_t* sm_off = m.off;
  const int32_t* sm_act = m.act;
  const int32_t* sm_tok = m.tok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hv = H / 8;
  // stage: [2][fr][H] weights, then [rcap][H] token rows of the item's expert
  const uint32_t wbytes = 2u * fr * H * 2;
  const uint32_t stage_bytes = wbytes + (uint32_t)rcap * H * 2;
  uint8_t* stage_base = dsm_raw;
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), kWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fence_proxy_async_smem();  // earlier generic use of this shared memory precedes the bulk copies
  const int nact = *m.nact;
  __syncthreads();
  const int nfc = (F + fr - 1) / fr;
  const int items = nact * nfc;
  const int mine = items > (int)bid ? (items - 1 - (int)bid) / (int)nblk + 1 : 0;
  auto issue = [&](int j) {
    const int item = bid + j * nblk;
    const int e = sm_act[item / nfc];
    const int f0 = (item % nfc) * fr;
    const int rows = min(fr, F - f0);
    const uint32_t bytes = (uint32_t)rows * H * 2;
    const int s = j % stages;
    const uint32_t dst = smem_u32(stage_base + (size_t)s * stage_bytes);
    const uint32_t bar = smem_u32(&full[s]);
    const int r0 = sm_off[e];
    const int rc = min(rcap, sm_off[e + 1] - r0);
    const uint32_t xrow = (uint32_t)H * 2;
    mbar_expect_tx(bar, 2 * bytes + rc * xrow);
    bulk_load(dst, w_gate + ((int64_t)e * F + f0) * H, bytes, bar);
    bulk_load(dst + (uint32_t)fr * H * 2, w_up + ((int64_t)e * F + f0) * H, bytes, bar);
    for (int r = 0; r < rc; ++r)
      bulk_load(dst + wbytes + r * xrow, x + (int64_t)sm_tok[r0 + r] * H, xrow, bar);
  };
  if (warp == kWarps) {
    // producer warp: refills a stage as soon as all compute warps released
    // it, so the compute warps never stall on issuing copies
    if (lane == 0)
      for (int j = 0; j < mine; ++j) {
        const int s = j % stages;
        if (j >= stages && !mbar_wait(smem_u32(&empty[s]), (uint32_t)(j / stages - 1) & 1u, s_abort, ws.err)) break;
        issue(j);
      }
    return;
  }
  for (int j = 0; j < mine; ++j) {
    const int item = bid + j * nblk;
    const int e = sm_act[item / nfc];
    const int f0 = (item % nfc) * fr;
    const int rows = min(fr, F - f0);
    const int s = j % stages;
    if (!mbar_wait(smem_u32(&full[s]), (uint32_t)(j / stages) & 1u, s_abort, ws.err)) break;
    const uint4* gsm = reinterpret_cast<const uint4*>(stage_base + (size_t)s * stage_bytes);
    const uint4* usm = gsm + (size_t)fr * hv;
    const int r0 = sm_off[e], cnt = sm_off[e + 1] - r0;
    for (int c0 = 0; c0 < cnt; c0 += rcap) {
      const int rc = min(rcap, cnt - c0);
      uint4* xr = reinterpret_cast<uint4*>(stage_base + (size_t)s * stage_bytes + wbytes);
      if (c0 > 0) {  // more than rcap rows: later chunks are gathered into the same area
        for (int i = threadIdx.x; i < rc * hv; i += kThreads) {
          const int r = i / hv, v = i - r * hv;
          xr[i] = reinterpret_cast<const uint4*>(x + (int64_t)sm_tok[r0 + c0 + r] * H)[v];
        }
        consumer_sync();
      }
      if (warp < rows) {
        const uint4* gr = gsm + (size_t)warp * hv;
        const uint4* ur = usm + (size_t)warp * hv;
        for (int r = 0; r < rc; ++r) {
          float g = 0.f, u = 0.f;
          // all shared-memory loads of a 256-slice round are issued before
          // any is used (independent loads instead of a dependent chain)
          for (int v0 = 0; v0 < hv; v0 += 32 * 8) {
            uint4 gq[8], uq[8], xq[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int v = v0 + lane + 32 * i;
              const bool ok = v < hv;
              gq[i] = ok ? gr[v] : make_uint4(0, 0, 0, 0);
              uq[i] = ok ? ur[v] : make_uint4(0, 0, 0, 0);
              xq[i] = ok ? xr[r * hv + v] : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float gv[8], uv[8], xv[8];
              bf16x8_to_f32(gq[i], gv);
              bf16x8_to_f32(uq[i], uv);
              bf16x8_to_f32(xq[i], xv);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                g = fmaf(gv[q], xv[q], g);
                u = fmaf(uv[q], xv[q], u);
              }
            }
          }
#pragma unroll
          for (int o = 16; o; o >>= 1) {
            g += __shfl_xor_sync(0xffffffffu, g, o);
            u += __shfl_xor_sync(0xffffffffu, u, o);
          }
          if (lane == 0) ws.hs[(int64_t)(r0 + c0 + r) * F + f0 + warp] = __float2bfloat16_rn(g * silu_ref(u));
        }
      }
      if (c0 + rcap < cnt) consumer_sync();  // the next chunk's rows overwrite xr
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&empty[s]));  // this warp is done with stage s
  }
}

__global__ void __launch_bounds__(kBlockThreads)
decode_gateup_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w_gate,
                     const __nv_bfloat16* __restrict__ w_up, int T, int H, int F, int E, int fr, int rcap, int stages,
                     DecodeWs ws) {
  extern __shared__ __align__(128) uint8_t dsm_raw[];
  __shared__ __align__(8) uint64_t full[4], empty[4];
  __shared__ int s_abort;
  if (threadIdx.x == 0) s_abort = 0;
  wait_prior_grid();
  allow_next_grid();
  __shared__ int32_t m_off[kMaxE + 1], m_act[kMaxE], m_nact, m_tok[kMaxSlots];
  __shared__ float m_w[kMaxSlots];
  const Meta m = load_meta(ws, T, E, m_off, m_act, &m_nact, m_tok, m_w);
  gateup_body(x, w_gate, w_up, T, H, F, E, fr, rcap, stages, ws, blockIdx.x, gridDim.x, dsm_raw, full, empty,
              &s_abort, m);
}

// down: item = (active expert e, hr rows of H starting at h0): stage =
// [hr][F] bf16.  Warp w computes rows h0 + w, h0 + w + 8, ...:
// d[row, h] = (down_e[h] . h_row) * gate weight of the row, fp32.
__device__ __forceinline__ void down_body(const __nv_bfloat16* __restrict__ w_down, int H, int F, int E, int hr,
                                          int rcap, int stages, DecodeWs ws, int bid, int nblk, uint8_t* dsm_raw,
                                          uint64_t* full, uint64_t* empty, int* s_abort, Meta m) {
  const int32_t* sm_off = m.off;
  const int32_t* sm_act = m.act;
  const float* sm_w = m.w;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int fv = F / 8;
  // stage: [hr][F] weights, then [rcap][F] h rows of the item's expert
  const uint32_t wbytes = (uint32_t)hr * F * 2;
  const uint32_t stage_bytes = wbytes + (uint32_t)rcap * F * 2;
  uint8_t* stage_base = dsm_raw;
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), kWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  fence_proxy_async_smem();  // earlier generic use of this shared memory precedes the bulk copies
  const int nact = *m.nact;
  __syncthreads();
  const int nhc = (H + hr - 1) / hr;
  const int items = nact * nhc;
  const int mine = items > (int)bid ? (items - 1 - (int)bid) / (int)nblk + 1 : 0;
  auto issue = [&](int j) {
    const int item = bid + j * nblk;
    const int e = sm_act[item / nhc];
    const int h0 = (item % nhc) * hr;
    const uint32_t bytes = (uint32_t)min(hr, H - h0) * F * 2;
    const int s = j % stages;
    const uint32_t bar = smem_u32(&full[s]);
    const int r0 = sm_off[e];
    const int rc = min(rcap, sm_off[e + 1] - r0);
    const uint32_t hbytes = (uint32_t)rc * F * 2;
    const uint32_t dst = smem_u32(stage_base + (size_t)s * stage_bytes);
    mbar_expect_tx(bar, bytes + hbytes);
    bulk_load(dst, w_down + ((int64_t)e * H + h0) * F, bytes, bar);
    bulk_load(dst + wbytes, ws.hs + (int64_t)r0 * F, hbytes, bar);
  };
  if (warp == kWarps) {
    // producer warp: refills a stage as soon as all compute warps released
    // it, so the compute warps never stall on issuing copies
    if (lane == 0)
      for (int j = 0; j < mine; ++j) {
        const int s = j % stages;
        if (j >= stages && !mbar_wait(smem_u32(&empty[s]), (uint32_t)(j / stages - 1) & 1u, s_abort, ws.err)) break;
        issue(j);
      }
    return;
  }
  for (int j = 0; j < mine; ++j) {
    const int item = bid + j * nblk;
    const int e = sm_act[item / nhc];
    const int h0 = (item % nhc) * hr;
    const int rows = min(hr, H - h0);
    const int s = j % stages;
    if (!mbar_wait(smem_u32(&full[s]), (uint32_t)(j / stages) & 1u, s_abort, ws.err)) break;
    const uint4* wsm = reinterpret_cast<const uint4*>(stage_base + (size_t)s * stage_bytes);
    const int r0 = sm_off[e], cnt = sm_off[e + 1] - r0;
    for (int c0 = 0; c0 < cnt; c0 += rcap) {
      const int rc = min(rcap, cnt - c0);
      uint4* hr8 = reinterpret_cast<uint4*>(stage_base + (size_t)s * stage_bytes + wbytes);
      if (c0 > 0) {  // more than rcap rows: later chunks are loaded into the same area
        for (int i = threadIdx.x; i < rc * fv; i += kThreads)
          hr8[i] = reinterpret_cast<const uint4*>(ws.hs + (int64_t)(r0 + c0) * F)[i];
        consumer_sync();
      }
      // each warp takes its rows jr = warp + 8*jj (jj < 4) together: four
      // independent dot products in flight
      for (int jb = 0; jb < rows; jb += 4 * kWarps) {
        for (int r = 0; r < rc; ++r) {
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          for (int v0 = 0; v0 < fv; v0 += 32 * 4) {
            uint4 hq[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int v = v0 + lane + 32 * i;
              hq[i] = v < fv ? hr8[r * fv + v] : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const int jr = jb + warp + kWarps * jj;
              const uint4* wr = wsm + (size_t)min(jr, rows - 1) * fv;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int v = v0 + lane + 32 * i;
                if (v < fv) {
                  float wv[8], hv8[8];
                  bf16x8_to_f32(wr[v], wv);
                  bf16x8_to_f32(hq[i], hv8);
#pragma unroll
                  for (int q = 0; q < 8; ++q) acc[jj] = fmaf(wv[q], hv8[q], acc[jj]);
                }
              }
            }
          }
#pragma unroll
          for (int o = 16; o; o >>= 1)
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) acc[jj] += __shfl_xor_sync(0xffffffffu, acc[jj], o);
          if (lane < 4) {
            const int jr = jb + warp + kWarps * lane;
            const float a = lane == 0 ? acc[0] : lane == 1 ? acc[1] : lane == 2 ? acc[2] : acc[3];
            if (jr < rows) {
              const int row = r0 + c0 + r;
              ws.d[(int64_t)row * H + h0 + jr] = a * sm_w[row];
            }
          }
        }
      }
      if (c0 + rcap < cnt) consumer_sync();  // the next chunk's rows overwrite the h area
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&empty[s]));  // this warp is done with stage s
  }
}

__global__ void __launch_bounds__(kBlockThreads)
decode_down_kernel(const __nv_bfloat16* __restrict__ w_down, int H, int F, int E, int hr, int rcap, int stages,
                   DecodeWs ws) {
  extern __shared__ __align__(128) uint8_t dsm_raw[];
  __shared__ __align__(8) uint64_t full[4], empty[4];
  __shared__ int s_abort;
  if (threadIdx.x == 0) s_abort = 0;
  wait_prior_grid();
  allow_next_grid();
  __shared__ int32_t m_off[kMaxE + 1], m_act[kMaxE], m_nact, m_tok[kMaxSlots];
  __shared__ float m_w[kMaxSlots];
  const Meta m = load_meta(ws, 1, E, m_off, m_act, &m_nact, m_tok, m_w);
  down_body(w_down, H, F, E, hr, rcap, stages, ws, blockIdx.x, gridDim.x, dsm_raw, full, empty, &s_abort, m);
}

// --------------------------------------------------------------- combine --
// y[t, h] = sum_{j<k} d[slot_pos[j*T + t], h] in slot order (deterministic).
template <class TY>
__device__ __forceinline__ void combine_body(int T, int H, int k, TY* y, const DecodeWs& ws, int64_t gtid,
                                             int64_t nthreads) {
  for (int64_t i = gtid; i < (int64_t)T * H; i += nthreads) {
    const int t = (int)(i / H), h = (int)(i - (int64_t)t * H);
    float acc = 0.f;
    for (int j = 0; j < k; ++j) acc += __ldcg(ws.d + (int64_t)__ldcg(ws.slot_pos + j * T + t) * H + h);
    if (ws.res) acc = ws.res[i] + acc;  // the sub-layer's residual add after the sum
    y[i] = from_f32<TY>(acc);
  }
}

template <class TY>
__global__ void __launch_bounds__(kThreads)
decode_combine_kernel(int T, int H, int k, TY* y, DecodeWs ws) {
  wait_prior_grid();
  combine_body<TY>(T, H, k, y, ws, (int64_t)blockIdx.x * kThreads + threadIdx.x, (int64_t)gridDim.x * kThreads);
}

// ---------------------------------------------------------- fused kernel --
// All phases in one cooperative launch (every block resident), separated by
// grid barriers, so the decode step pays one launch and no inter-kernel gaps.  The barrier spins on a counter for at most ~2 s; on
// expiry it records FRANK_ETIMEOUT and lets the kernel run to its end.
__device__ __forceinline__ void grid_barrier(unsigned* counter, unsigned target, int* s_abort, int32_t* err) {
  asm volatile("fence.proxy.async.global;" ::: "memory");  // generic writes before later bulk reads
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    atomicAdd(counter, 1u);
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counter) : "memory");
      if (v >= target) break;
      if ((i & 63u) == 63u) {
        const uint64_t now = global_ns();
        if (t0 == 0) {
          t0 = now;
        } else if (now - t0 > 2000000000ull) {
          atomicExch(err, FRANK_ETIMEOUT);
          *s_abort = 1;
          break;
        }
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
}

// Dynamic shared memory of the fused kernel's routing phases: prob [T][E]
// f32, the block's top-k weights / ids [kMaxSlots], the permute scratch.
size_t fused_routing_smem(int64_t T, int64_t E) {
  return (size_t)((T * E * 4 + 15) / 16) * 16 + (sizeof(float) + sizeof(int32_t)) * kMaxSlots + kFinalizeSmem;
}
struct FusedRoutingSmem {
  float* prob;
  float* w;
  int32_t* ids;
  uint8_t* scratch;
};
__device__ __forceinline__ FusedRoutingSmem carve_fused_routing(uint8_t* base, int T, int E) {
  FusedRoutingSmem r;
  r.prob = reinterpret_cast<float*>(base);
  r.w = reinterpret_cast<float*>(base + (((size_t)T * E * 4 + 15) / 16) * 16);
  r.ids = reinterpret_cast<int32_t*>(r.w + kMaxSlots);
  r.scratch = reinterpret_cast<uint8_t*>(r.ids + kMaxSlots);
  return r;
}

template <class TW, class TY>
__global__ void __launch_bounds__(kBlockThreads, 1)
decode_fused_kernel(const __nv_bfloat16* __restrict__ x, const TW* __restrict__ wr,
                    const __nv_bfloat16* __restrict__ w_gate, const __nv_bfloat16* __restrict__ w_up,
                    const __nv_bfloat16* __restrict__ w_down, int T, int H, int F, int E, int k, int normalize,
                    int fr, int stages_gu, int hr, int stages_dn, int rcap, TY* y, DecodeWs ws) {
  extern __shared__ __align__(128) uint8_t dsm_raw[];
  __shared__ __align__(8) uint64_t full_gu[4], full_dn[4], empty_gu[4], empty_dn[4];
  __shared__ int s_abort;
  if (threadIdx.x == 0) s_abort = 0;
  const int bid = blockIdx.x, nblk = gridDim.x;
  const bool compute = threadIdx.x < kThreads;  // warps 0..kWarps-1; the last warp produces copies
  if (compute) route_body<TW>(x, wr, T, H, E, ws, reinterpret_cast<float*>(dsm_raw), bid, nblk);
  grid_barrier(ws.gbar, 1u * nblk, &s_abort, ws.err);
  // every block runs softmax / top-k for all T tokens and builds the (small)
  // permutation itself, so the streaming phases start without another
  // barrier; block 0 also publishes the routing
  __shared__ int32_t m_off[kMaxE + 1], m_act[kMaxE], m_nact, m_tok[kMaxSlots];
  __shared__ float m_w[kMaxSlots];
  const Meta m{m_off, m_act, &m_nact, m_tok, m_w};
  if (compute) {
    const FusedRoutingSmem rs = carve_fused_routing(dsm_raw, T, E);
    block_softmax_topk(ws.logits, T, E, k, normalize, rs.prob, rs.w, rs.ids);
    if (bid == 0)
      for (int i = threadIdx.x; i < k * T; i += kThreads) {
        ws.w[i] = rs.w[i];
        ws.ids[i] = rs.ids[i];
      }
    if (k * T <= 32)
      small_permute_body(T, E, k, ws, m, rs.ids, rs.w, bid == 0);
    else
      permute_body(T, E, k, ws, rs.scratch, m, rs.ids, rs.w, bid == 0);
  }
  __syncthreads();  // the routing tables, for the producer warp too
  gateup_body(x, w_gate, w_up, T, H, F, E, fr, rcap, stages_gu, ws, bid, nblk, dsm_raw, full_gu, empty_gu, &s_abort,
              m);
  grid_barrier(ws.gbar, 2u * nblk, &s_abort, ws.err);
  down_body(w_down, H, F, E, hr, rcap, stages_dn, ws, bid, nblk, dsm_raw, full_dn, empty_dn, &s_abort, m);
  grid_barrier(ws.gbar, 3u * nblk, &s_abort, ws.err);
  if (compute) combine_body<TY>(T, H, k, y, ws, (int64_t)bid * kThreads + threadIdx.x, (int64_t)nblk * kThreads);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

template <class TW, class TY>
int launch_fused(const void* x, const void* wr, const void* wg, const void* wu, const void* wd, int64_t T, int64_t H,
                 int64_t F, int64_t E, int64_t k, int normalize, int fr, int stages_gu, int hr, int stages_dn,
                 int rcap, void* y, const DecodeWs& ws, size_t smem, cudaStream_t st) {
  auto kern = decode_fused_kernel<TW, TY>;
  FRANK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  FRANK_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kBlockThreads, smem));
  if (per_sm < 1) {
    frank::set_error("decode block: the fused kernel does not fit on an SM");
    return FRANK_EINVAL;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(frank::num_sms());
  cfg.blockDim = dim3(kBlockThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FRANK_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, (const __nv_bfloat16*)x, (const TW*)wr, (const __nv_bfloat16*)wg,
                                    (const __nv_bfloat16*)wu, (const __nv_bfloat16*)wd, (int)T, (int)H, (int)F,
                                    (int)E, (int)k, normalize, fr, stages_gu, hr, stages_dn, rcap, (TY*)y, ws));
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

// Shared-memory staging of the two streaming phases.  An expert receives at
// most T rows (the top-k ids of a token are distinct), so a stage holds
// rcap = min(kRC, T) token rows beside its weights.  Rows per item start at
// 32 KB of each gate/up matrix and 48 KB of down and halve until two stages
// fit; a shape where even one row does not leaves the decode path.
struct DecodePlan {
  int rcap, fr, hr, stages_gu, stages_dn;
  size_t stage_gu, stage_dn;
  bool ok;
};

DecodePlan decode_plan(int64_t T, int64_t H, int64_t F) {
  // dynamic shared memory beside the kernels' static tables (< 8 KB)
  constexpr size_t kSmemDyn = 227 * 1024 - 8 * 1024;
  DecodePlan p{};
  p.rcap = (int)(T < kRC ? T : kRC);
  p.fr = (int)(16384 / H < 1 ? 1 : (16384 / H > kWarps ? kWarps : 16384 / H));
  p.hr = (int)(24576 / F < 1 ? 1 : (24576 / F > 32 ? 32 : 24576 / F));
  for (;;) {
    p.stage_gu = (size_t)2 * p.fr * H * 2 + (size_t)p.rcap * H * 2;
    p.stages_gu = (int)(kSmemDyn / p.stage_gu);
    if (p.stages_gu >= 2 || p.fr == 1) break;
    p.fr /= 2;
  }
  for (;;) {
    p.stage_dn = (size_t)p.hr * F * 2 + (size_t)p.rcap * F * 2;
    p.stages_dn = (int)(kSmemDyn / p.stage_dn);
    if (p.stages_dn >= 2 || p.hr == 1) break;
    p.hr /= 2;
  }
  // about 96 KB in flight per SM is enough to stream at full rate; deeper
  // rings only add shared-memory write traffic that slows the dot products
  // of the stage being consumed (measured: T=1 with 3-4 stages of 49-68 KB,
  // 45 us; 2 stages, 43 us)
  auto depth = [](size_t stage) {
    const int want = (int)((96 * 1024 + stage - 1) / stage);
    return want < 2 ? 2 : (want > 4 ? 4 : want);
  };
  p.stages_gu = p.stages_gu > depth(p.stage_gu) ? depth(p.stage_gu) : p.stages_gu;
  p.stages_dn = p.stages_dn > depth(p.stage_dn) ? depth(p.stage_dn) : p.stages_dn;
  p.ok = p.stages_gu >= 2 && p.stages_dn >= 2;
  return p;
}

}  // namespace

namespace frank {

bool decode_path_ok(int dtype, int64_t T, int64_t H, int64_t F, int64_t E, int64_t k) {
  return dtype == FRANK_BF16 && T >= 1 && T <= 64 && k * T <= kMaxSlots && E <= kMaxE && H % 8 == 0 && F % 8 == 0 &&
         k * T <= E && decode_plan(T, H, F).ok;
}

size_t decode_workspace_size(int64_t T, int64_t H, int64_t F, int64_t E, int64_t k) {
  Carve c(nullptr, 0);
  const int64_t n = k * T;
  c.take<float>(E * T);
  c.take<float>(n);
  c.take<int32_t>(n);
  c.take<int32_t>(n);
  c.take<int32_t>(E + 1);
  c.take<int32_t>(n);
  c.take<float>(n);
  c.take<__nv_bfloat16>(n * F);
  c.take<int32_t>(E);
  c.take<int32_t>(1);
  c.take<float>(n * H);
  c.take<unsigned>(1);
  return align_up(c.used, 256);
}

// Writes route_w / route_ids when non-null (copies of the internal buffers).
int launch_decode_block(const void* x, int wr_dtype, const void* wr, const void* w_up_p, const void* w_gate_p,
                        const void* w_down_p, int64_t T, int64_t E, int64_t k, int64_t H, int64_t F, int normalize,
                        int y_dtype, void* y, float* route_w, int32_t* route_ids, void* workspace, size_t ws_bytes,
                        cudaStream_t st, void (*mark)(int, cudaStream_t), const float* residual) {
  if (ws_bytes < decode_workspace_size(T, H, F, E, k)) {
    set_error("decode block: workspace %zu < %zu", ws_bytes, decode_workspace_size(T, H, F, E, k));
    return FRANK_ENOSPC;
  }
  if ((uintptr_t)x % 16 || (uintptr_t)w_up_p % 16 || (uintptr_t)w_gate_p % 16 || (uintptr_t)w_down_p % 16 ||
      (uintptr_t)wr % 16) {
    set_error("decode block: inputs must be 16-byte aligned");
    return FRANK_EINVAL;
  }
  const int64_t n = k * T;
  Carve c(workspace, ws_bytes);
  DecodeWs ws;
  ws.logits = c.take<float>(E * T);
  ws.w = c.take<float>(n);
  ws.ids = c.take<int32_t>(n);
  ws.sorted_slots = c.take<int32_t>(n);
  ws.offsets = c.take<int32_t>(E + 1);
  ws.slot_pos = c.take<int32_t>(n);
  ws.wsorted = c.take<float>(n);
  ws.hs = c.take<__nv_bfloat16>(n * F);
  ws.active = c.take<int32_t>(E);
  ws.nactive = c.take<int32_t>(1);
  ws.d = c.take<float>(n * H);
  ws.gbar = c.take<unsigned>(1);
  ws.res = residual;
  ws.n_slots = (int)n;
  ws.err = device_error_word();
  const DecodePlan plan = decode_plan(T, H, F);
  if (!plan.ok) {
    set_error("decode block: n_embd=%lld / n_ff=%lld too large for the streaming kernels", (long long)H,
              (long long)F);
    return FRANK_EINVAL;
  }
  const int rcap = plan.rcap, fr = plan.fr, hr = plan.hr, stages_gu = plan.stages_gu, stages_dn = plan.stages_dn;
  const size_t stage_gu = plan.stage_gu, stage_dn = plan.stage_dn;
  const char* fenv = getenv("FRANK_DECODE_FUSED");
  if (!(fenv && fenv[0] == '0')) {
    // one cooperative launch (decode_fused_kernel)
    size_t smem = stages_gu * stage_gu;
    if (stages_dn * stage_dn > smem) smem = stages_dn * stage_dn;
    if (fused_routing_smem(T, E) > smem) smem = fused_routing_smem(T, E);
    mark(0, st);
    FRANK_CUDA_TRY(cudaMemsetAsync(ws.gbar, 0, sizeof(unsigned), st));
    int st_launch;
    if (wr_dtype == FRANK_F32 && y_dtype == FRANK_F32)
      st_launch = launch_fused<float, float>(x, wr, w_gate_p, w_up_p, w_down_p, T, H, F, E, k, normalize, fr,
                                             stages_gu, hr, stages_dn, rcap, y, ws, smem, st);
    else if (wr_dtype == FRANK_F32)
      st_launch = launch_fused<float, __nv_bfloat16>(x, wr, w_gate_p, w_up_p, w_down_p, T, H, F, E, k, normalize, fr,
                                                     stages_gu, hr, stages_dn, rcap, y, ws, smem, st);
    else if (y_dtype == FRANK_F32)
      st_launch = launch_fused<__nv_bfloat16, float>(x, wr, w_gate_p, w_up_p, w_down_p, T, H, F, E, k, normalize, fr,
                                                     stages_gu, hr, stages_dn, rcap, y, ws, smem, st);
    else
      st_launch = launch_fused<__nv_bfloat16, __nv_bfloat16>(x, wr, w_gate_p, w_up_p, w_down_p, T, H, F, E, k,
                                                             normalize, fr, stages_gu, hr, stages_dn, rcap, y, ws,
                                                             smem, st);
    FRANK_TRY(st_launch);
    for (int m = 1; m <= 6; ++m) mark(m, st);
  } else {
  mark(0, st);
  const unsigned rblocks = (unsigned)num_sms();
  if (wr_dtype == FRANK_F32)
    decode_route_kernel<float><<<rblocks, kThreads, 0, st>>>((const __nv_bfloat16*)x, (const float*)wr, (int)T,
                                                             (int)H, (int)E, (int)k, normalize, ws);
  else
    decode_route_kernel<__nv_bfloat16><<<rblocks, kThreads, 0, st>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)wr, (int)T, (int)H, (int)E, (int)k, normalize, ws);
  FRANK_LAUNCH_CHECK();
  const size_t prob_smem = (size_t)T * E * sizeof(float);
  FRANK_CUDA_TRY(cudaFuncSetAttribute(decode_finalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)prob_smem));
  FRANK_CUDA_TRY(launch_pdl(decode_finalize_kernel, dim3(1), dim3(kThreads), prob_smem, st, (int)T, (int)E, (int)k,
                            normalize, ws));
  FRANK_LAUNCH_CHECK();
  mark(1, st);
  mark(2, st);
  mark(3, st);
  ws.err = device_error_word();
  const int grid_p = num_sms();
  {
    const size_t smem = stages_gu * stage_gu;
    FRANK_CUDA_TRY(cudaFuncSetAttribute(decode_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    FRANK_CUDA_TRY(launch_pdl(decode_gateup_kernel, dim3(grid_p), dim3(kBlockThreads), smem, st,
                              (const __nv_bfloat16*)x, (const __nv_bfloat16*)w_gate_p,
                              (const __nv_bfloat16*)w_up_p, (int)T, (int)H, (int)F, (int)E, fr, rcap, stages_gu,
                              ws));
    FRANK_LAUNCH_CHECK();
  }
  mark(4, st);
  {
    const size_t smem = stages_dn * stage_dn;
    FRANK_CUDA_TRY(cudaFuncSetAttribute(decode_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    FRANK_CUDA_TRY(launch_pdl(decode_down_kernel, dim3(grid_p), dim3(kBlockThreads), smem, st,
                              (const __nv_bfloat16*)w_down_p, (int)H, (int)F, (int)E, hr, rcap, stages_dn, ws));
    FRANK_LAUNCH_CHECK();
  }
  mark(5, st);
  {
    const int64_t tot = T * H;
    const unsigned g = (unsigned)((tot + kThreads - 1) / kThreads);
    if (y_dtype == FRANK_F32)
      FRANK_CUDA_TRY(launch_pdl(decode_combine_kernel<float>, dim3(g), dim3(kThreads), 0, st, (int)T, (int)H,
                                (int)k, (float*)y, ws));
    else
      FRANK_CUDA_TRY(launch_pdl(decode_combine_kernel<__nv_bfloat16>, dim3(g), dim3(kThreads), 0, st, (int)T,
                                (int)H, (int)k, (__nv_bfloat16*)y, ws));
    FRANK_LAUNCH_CHECK();
  }
  mark(6, st);
  }
  if (route_w) FRANK_CUDA_TRY(cudaMemcpyAsync(route_w, ws.w, n * sizeof(float), cudaMemcpyDeviceToDevice, st));
  if (route_ids)
    FRANK_CUDA_TRY(cudaMemcpyAsync(route_ids, ws.ids, n * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  return FRANK_OK;
}

}  // namespace frank
