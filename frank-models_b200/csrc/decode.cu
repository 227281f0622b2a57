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
//   gate/up  the (gate row, up row) pairs of the active experts split evenly
//            over persistent blocks, in items of up to fr rows of one
//            expert: the rows streamed once into shared memory with bulk
//            copies and dotted with the expert's token rows (gathered
//            straight from x), h = gate * silu(up) (swiglu.mlir:37-47);
//   down     block b owns the output columns [b H / nblk, (b+1) H / nblk)
//            of every token and streams those rows of every active expert's
//            down matrix: d = down(h) * gate weight, fp32, kept in shared
//            memory; then y[t] = sum of the k slots of t in slot order
//            (moe_ffn_block.mlir:179-206) for its columns, deterministic.
// decode_fused_kernel runs all phases in one cooperative launch with two
// grid barriers (after route and after gate/up): every block computes the
// top-k and the permutation of all tokens itself, and requests its first
// down weight rows before the second barrier.  Blocks have eight compute
// warps plus one warp that issues the streaming phases' bulk copies.
// FRANK_DECODE_FUSED=0 runs the same bodies as four launches chained by
// programmatic dependent launch.  No atomics on data: results are
// deterministic and identical in both forms.
#include <cstdlib>

#include "common.cuh"
#include "mbarrier.cuh"
#include "topk.cuh"

namespace {

using namespace frank_topk;
using frank::align_up;

#ifdef FRANK_DECODE_TRACE
// Measurement builds only: %globaltimer at the phase boundaries of every
// block of the last fused launch (read with frank_decode_trace_read).
__device__ unsigned long long g_decode_trace[1024][8];
// per-item trace of block 0: [phase 0 gate/up, 1 down][item][landed, done, issued]
__device__ unsigned long long g_decode_items[2][64][3];
#define TRACE_ITEM(ph, j, w)                                                        \
  do {                                                                              \
    if (blockIdx.x == 0 && (j) < 64) g_decode_items[ph][j][w] = frank_mbar::global_ns(); \
  } while (0)
#define TRACE(i)                                                         \
  do {                                                                   \
    if (threadIdx.x == 0) g_decode_trace[blockIdx.x][i] = frank_mbar::global_ns();   \
  } while (0)
#else
#define TRACE(i) \
  do {           \
  } while (0)
#define TRACE_ITEM(ph, j, w) \
  do {                       \
  } while (0)
#endif


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
  int32_t* err;         // device error word (bounded waits)
  unsigned* gbar;       // [2] grid-barrier and exit counters of the fused kernel (zero between calls)
  const float* res;     // optional fp32 [T, H] residual added to y (may alias y)
  int n_slots;          // k * T
};

// Routing tables of one call in shared memory: expert row offsets [E+1],
// active experts [E] (first *nact valid), token of each expert-sorted row,
// gate weight of each expert-sorted row, expert-sorted row of each flat
// slot s = j*T + t.
struct Meta {
  int32_t* off;
  int32_t* act;
  int32_t* nact;
  int32_t* tok;
  float* w;
  int32_t* pos;
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
constexpr int kPerLane = kMaxE / 32;

// The selection steps on one token's probabilities held in registers
// (p[i] = probability of expert lane + 32 i, -1 where absent).
__device__ __forceinline__ void warp_topk_select(float (&p)[kPerLane], int k, int normalize, float* w_out,
                                                 int32_t* id_out, int T, int t) {
  const int lane = threadIdx.x & 31;
  constexpr int kPer = kPerLane;
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

__device__ __forceinline__ void warp_softmax_topk_probs(const float* p_in, int E, int k, int normalize, float* w_out,
                                                        int32_t* id_out, int T, int t) {
  const int lane = threadIdx.x & 31;
  float p[kPerLane];
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? p_in[e] : -1.f;  // probabilities are >= 0; -1 marks "absent"
  }
  warp_topk_select(p, k, normalize, w_out, id_out, T, t);
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
  if (T <= kWarps) {
    // one warp per token, probabilities kept in registers: no shared-memory
    // round trip and one barrier (same arithmetic and selection as below)
    if (warp < T) {
      const int t = warp;
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
      for (int i = 0; i < kPer; ++i) v[i] = lane + 32 * i < E ? v[i] / sum : -1.f;
      warp_topk_select(v, k, normalize, w_out, id_out, T, t);
    }
    consumer_sync();
    return;
  }
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
    m.pos[s] = pos;
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
      m.pos[lane] = pos;
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
  __shared__ int32_t m_pos[kMaxSlots];
  wait_prior_grid();
  allow_next_grid();
  finalize_body(T, E, k, normalize, ws, scratch, prob, Meta{m_off, m_act, &m_nact, m_tok, m_w, m_pos});
}


__device__ __forceinline__ Meta load_meta(const DecodeWs& ws, int T, int E, int32_t* off, int32_t* act, int32_t* nact,
                                          int32_t* tok, float* w, int32_t* pos) {
  for (int i = threadIdx.x; i <= E; i += blockDim.x) off[i] = __ldcg(ws.offsets + i);
  for (int i = threadIdx.x; i < E; i += blockDim.x) act[i] = __ldcg(ws.active + i);
  for (int i = threadIdx.x; i < ws.n_slots; i += blockDim.x) {
    tok[i] = __ldcg(ws.sorted_slots + i) % T;
    w[i] = __ldcg(ws.wsorted + i);
    pos[i] = __ldcg(ws.slot_pos + i);
  }
  if (threadIdx.x == 0) *nact = __ldcg(ws.nactive);
  __syncthreads();
  return Meta{off, act, nact, tok, w, pos};
}

// ----------------------------------------------- weight-streaming GEMVs --
// Both GEMV kernels stream contiguous chunks of an expert's weight rows from
// HBM into a ring of shared-memory stages with 1-D bulk copies
// (cp.async.bulk, one mbarrier per stage), so that every SM keeps 100+ KB of
// weights in flight; the token rows of the chunk's expert are staged next to
// them and every warp dots whole rows out of shared memory.  Items are
// (active expert, chunk of rows), spread over persistent blocks.
using namespace frank_mbar;

// Barriers of a streaming ring: full (one producer arrival + the bytes),
// empty (one arrival per compute warp).
__device__ __forceinline__ void init_ring(uint64_t* full, uint64_t* empty, int stages) {
  for (int i = 0; i < stages; ++i) {
    mbar_init(smem_u32(&full[i]), 1);
    mbar_init(smem_u32(&empty[i]), kWarps);
  }
}


// ------------------------------------------------ tensor-core dot products --
// The streaming phases multiply a few weight rows by a few token rows: a
// 16 x 8 output tile over K, i.e. warp MMAs m16n8k16 (bf16 in, fp32
// accumulate).  The weight rows arrive by one contiguous bulk copy, so 16
// rows sit at a stride of K * 2 bytes.  Instead of ldmatrix (whose 8 rows of
// one 8 x 8 matrix would then share a bank group) each thread loads 16
// contiguous bytes per row with one 128-bit load: thread t of a quad takes
// the physical K elements [8t, 8t + 8) of every 32-element block and feeds
// them to the fragment slots of logical k {2t, 2t+1, 2t+8, 2t+9} of the
// block's two MMAs.  A and B use the same physical-to-logical map (it depends
// on t only), so each output is still the full dot product.  The K blocks are
// split evenly over the compute warps and their partial tiles summed in warp
// order (deterministic).
__host__ __device__ inline uint32_t tok_stride(int K) { return (uint32_t)K * 2 + 64; }
constexpr int kMT = 16;  // weight rows per tile

__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// This warp's share of A [16 x K] times the token rows B^T [nb x K] (row n
// at b + n * brs, n < nb <= 8), written to red[warp] as a [16][8] tile.
// A's rows 0..7 are the rows i < nlo at lo + i * ars, its rows 8..15 the
// rows i - 8 < nhi at hi + (i - 8) * ars; rows beyond nlo / nhi, like token
// columns beyond nb, repeat the last row and their outputs are ignored (so
// a stage only holds the rows it uses).  K % 16 == 0.
__device__ __forceinline__ void warp_tile_mma(const uint8_t* lo, int nlo, const uint8_t* hi, int nhi, uint32_t ars,
                                              const uint8_t* b, uint32_t brs, int K, int nb, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int full = K / 32;
  const int units = full + ((K & 31) ? 1 : 0);
  const int u0 = units * warp / kWarps, u1 = units * (warp + 1) / kWarps;
  const uint8_t* ap0 = lo + (size_t)min(g, max(nlo - 1, 0)) * ars;
  const uint8_t* ap1 = hi + (size_t)min(g, max(nhi - 1, 0)) * ars;
  const uint8_t* bp = b + (size_t)min(g, nb - 1) * brs;
  // four independent accumulators, each group's loads issued before its MMAs
  float acc[4][4];
#pragma unroll
  for (int q = 0; q < 4; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
  const int uf = min(u1, full);
  for (int ub = u0; ub < uf; ub += 4) {
    uint4 A0[4], A1[4], B[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (ub + q < uf) {
        const int off = (ub + q) * 64 + t * 16;
        A0[q] = *reinterpret_cast<const uint4*>(ap0 + off);
        A1[q] = *reinterpret_cast<const uint4*>(ap1 + off);
        B[q] = *reinterpret_cast<const uint4*>(bp + off);
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (ub + q < uf) {
        mma_16816(acc[q], A0[q].x, A1[q].x, A0[q].y, A1[q].y, B[q].x, B[q].y);
        mma_16816(acc[q], A0[q].z, A1[q].z, A0[q].w, A1[q].w, B[q].z, B[q].w);
      }
    }
  }
  if (u1 > full) {  // the last 16 elements: physical [4t, 4t + 4) for logical {2t, 2t+1, 2t+8, 2t+9}
    const int off = full * 64 + t * 8;
    const uint2 A0 = *reinterpret_cast<const uint2*>(ap0 + off);
    const uint2 A1 = *reinterpret_cast<const uint2*>(ap1 + off);
    const uint2 B = *reinterpret_cast<const uint2*>(bp + off);
    mma_16816(acc[0], A0.x, A1.x, A0.y, A1.y, B.x, B.y);
  }
  float c[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = ((acc[0][i] + acc[1][i]) + acc[2][i]) + acc[3][i];
  // m16n8 accumulator: c0, c1 at (g, 2t + {0, 1}), c2, c3 at (g + 8, 2t + {0, 1})
  float* o = red + warp * (kMT * 8);
  o[g * 8 + 2 * t] = c[0];
  o[g * 8 + 2 * t + 1] = c[1];
  o[(g + 8) * 8 + 2 * t] = c[2];
  o[(g + 8) * 8 + 2 * t + 1] = c[3];
}

// sum over the warps' partial tiles, in warp order
__device__ __forceinline__ float red_sum(const float* red, int i, int n) {
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) s += red[w * (kMT * 8) + i * 8 + n];
  return s;
}

// gate/up: the nact * F (gate row, up row) pairs of the active experts are
// split evenly over the blocks -- block b takes the flat pairs
// [b R / nblk, (b+1) R / nblk), R = nact * F -- and a block walks its range in
// items of at most fr <= 8 consecutive rows of one expert (an item ends at an
// expert boundary).  Stage = the item's gate rows, then its up rows (one
// bulk copy each, fr rows reserved for each) and the expert's token rows.
// One 16 x 8 tile gives gate . x and up . x of every (row, token):
// h = gate . x * silu(up . x).
struct GuCursor {
  int64_t c, hi;  // next flat pair, end of this block's range
  int F, fr;
  __device__ __forceinline__ bool next(int& a, int& f0, int& rows) {
    if (c >= hi) return false;
    a = (int)(c / F);
    f0 = (int)(c - (int64_t)a * F);
    rows = (int)min((int64_t)min(fr, F - f0), hi - c);
    c += rows;
    return true;
  }
};

__device__ __forceinline__ GuCursor gu_range(int nact, int F, int fr, int bid, int nblk) {
  const int64_t R = (int64_t)nact * F;
  return GuCursor{R * bid / nblk, R * (bid + 1) / nblk, F, fr};
}

__device__ __host__ inline uint32_t gu_stage_bytes(int H, int fr, int rcap) {
  return (uint32_t)(2 * fr) * H * 2 + (uint32_t)rcap * tok_stride(H);
}

__device__ __forceinline__ void gateup_body(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w_gate,
                     const __nv_bfloat16* __restrict__ w_up, int T, int H, int F, int E, int fr, int rcap, int stages,
                     DecodeWs ws, int bid, int nblk, uint8_t* dsm_raw, float* red, uint64_t* full, uint64_t* empty,
                     int* s_abort, Meta m) {
  // routing tables in shared memory: refilling a stage needs no global round trip
  const int32_t* sm_off = m.off;
  const int32_t* sm_act = m.act;
  const int32_t* sm_tok = m.tok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t xrow = (uint32_t)H * 2;  // weight row stride
  const uint32_t ts = tok_stride(H);      // token row stride
  const uint32_t stage_bytes = gu_stage_bytes(H, fr, rcap);
  uint8_t* stage_base = dsm_raw;
  const int nact = *m.nact;
  if (warp == kWarps) {
    // producer warp: refills a stage as soon as all compute warps released
    // it, so the compute warps never stall on issuing copies
    if (lane == 0) {
      fence_proxy_async_smem();  // earlier generic use of this shared memory precedes the bulk copies
      GuCursor cur = gu_range(nact, F, fr, bid, nblk);
      int a, f0, rows;
      for (int j = 0; cur.next(a, f0, rows); ++j) {
        const int s = j % stages;
        if (j >= stages && !mbar_wait(smem_u32(&empty[s]), (uint32_t)(j / stages - 1) & 1u, s_abort, ws.err)) break;
        TRACE_ITEM(0, j, 2);
        const int e = sm_act[a];
        const uint32_t dst = smem_u32(stage_base + (size_t)s * stage_bytes);
        const uint32_t bar = smem_u32(&full[s]);
        const int r0 = sm_off[e];
        const int rc = min(rcap, sm_off[e + 1] - r0);
        mbar_expect_tx(bar, (uint32_t)(2 * rows + rc) * xrow);
        bulk_load(dst, w_gate + ((int64_t)e * F + f0) * H, (uint32_t)rows * xrow, bar);
        bulk_load(dst + fr * xrow, w_up + ((int64_t)e * F + f0) * H, (uint32_t)rows * xrow, bar);
        for (int r = 0; r < rc; ++r)
          bulk_load(dst + 2 * fr * xrow + r * ts, x + (int64_t)sm_tok[r0 + r] * H, xrow, bar);
      }
    }
    return;
  }
  GuCursor cur = gu_range(nact, F, fr, bid, nblk);
  int a, f0, rows, tile = 0;
  for (int j = 0; cur.next(a, f0, rows); ++j) {
    const int e = sm_act[a];
    const int s = j % stages;
    if (!mbar_wait(smem_u32(&full[s]), (uint32_t)(j / stages) & 1u, s_abort, ws.err)) break;
    if (threadIdx.x == 0) TRACE_ITEM(0, j, 0);
    uint8_t* st = stage_base + (size_t)s * stage_bytes;
    uint8_t* tok = st + 2 * fr * xrow;
    const int r0 = sm_off[e], cnt = sm_off[e + 1] - r0;
    for (int c0 = 0; c0 < cnt; c0 += rcap) {
      const int rc = min(rcap, cnt - c0);
      if (c0 > 0) {  // more than rcap token rows: later chunks are gathered into the same area
        const int hv = H / 8;
        for (int i = threadIdx.x; i < rc * hv; i += kThreads) {
          const int r = i / hv, v = i - r * hv;
          *reinterpret_cast<uint4*>(tok + r * ts + v * 16) =
              reinterpret_cast<const uint4*>(x + (int64_t)sm_tok[r0 + c0 + r] * H)[v];
        }
        consumer_sync();
      }
      // partial tiles alternate between two buffers: one barrier per tile
      float* rb = red + (tile++ & 1) * (kWarps * kMT * 8);
      warp_tile_mma(st, rows, st + fr * xrow, rows, xrow, tok, ts, H, rc, rb);
      if (c0 + rcap >= cnt) {
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&empty[s]));  // this warp is done with stage s
      }
      consumer_sync();
      if (threadIdx.x < 64) {
        const int i = threadIdx.x >> 3, n = threadIdx.x & 7;
        if (i < rows && n < rc) {
          const float g = red_sum(rb, i, n), u = red_sum(rb, i + 8, n);
          ws.hs[(int64_t)(r0 + c0 + n) * F + f0 + i] = __float2bfloat16_rn(g * silu_ref(u));
        }
      }
      if (c0 + rcap < cnt) consumer_sync();  // the next chunk's rows overwrite the token area
    }
    if (threadIdx.x == 0) TRACE_ITEM(0, j, 1);
  }
}

__global__ void __launch_bounds__(kBlockThreads)
decode_gateup_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w_gate,
                     const __nv_bfloat16* __restrict__ w_up, int T, int H, int F, int E, int fr, int rcap, int stages,
                     DecodeWs ws) {
  extern __shared__ __align__(128) uint8_t dsm_raw[];
  __shared__ __align__(8) uint64_t full[4], empty[4];
  __shared__ __align__(16) float red[2 * kWarps * kMT * 8];
  __shared__ int s_abort;
  if (threadIdx.x == 0) {
    s_abort = 0;
    init_ring(full, empty, stages);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  wait_prior_grid();
  allow_next_grid();
  __shared__ int32_t m_off[kMaxE + 1], m_act[kMaxE], m_nact, m_tok[kMaxSlots], m_pos[kMaxSlots];
  __shared__ float m_w[kMaxSlots];
  const Meta m = load_meta(ws, T, E, m_off, m_act, &m_nact, m_tok, m_w, m_pos);
  gateup_body(x, w_gate, w_up, T, H, F, E, fr, rcap, stages, ws, blockIdx.x, gridDim.x, dsm_raw, red, full, empty,
              &s_abort, m);
}

// down + combine: block b owns the output columns [hb0, hb1) = [b H / nblk,
// (b+1) H / nblk) of y for every token.  Its items are (active expert e,
// at most hr <= 16 rows of its columns starting at h0); block b starts at
// active expert b mod nact, so the blocks read different experts' rows at
// the same time.  Stage = up to 16 rows of down_e (one bulk copy), then the
// expert's h rows.  One 16 x 8 tile per item: d[row, h] = (down_e[h] .
// h_row) * gate weight of the row, kept in shared memory (dsm [slots][nhmax]
// fp32, by expert-sorted row).  After the last item the block sums the k
// slots of each token in slot order j = 0..k-1 (moe_ffn_block.mlir:179-206),
// adds the residual when there is one, and writes y[:, hb0:hb1): no global d
// buffer, no combine pass and no barrier after the down rows.
//
// The first `pre` items' weight rows were already requested by
// down_prefetch (before the grid barrier that publishes h); for those the
// producer only adds the h rows to the stage.
struct DnCursor {
  int i, start, h0, nact, hb0, hb1, hr;
  __device__ __forceinline__ bool next(int& ea, int& eh0, int& rows) {
    if (i >= nact || hb0 >= hb1) return false;
    ea = start + i < nact ? start + i : start + i - nact;
    eh0 = h0;
    rows = min(hr, hb1 - h0);
    h0 += rows;
    if (h0 >= hb1) {
      h0 = hb0;
      ++i;
    }
    return true;
  }
};

__device__ __forceinline__ DnCursor dn_range(int nact, int H, int hr, int bid, int nblk) {
  const int hb0 = (int)((int64_t)H * bid / nblk), hb1 = (int)((int64_t)H * (bid + 1) / nblk);
  return DnCursor{0, nact > 0 ? bid % nact : 0, hb0, nact, hb0, hb1, hr};
}

__device__ __host__ inline uint32_t dn_stage_bytes(int F, int hr, int rcap) {
  return (uint32_t)hr * F * 2 + (uint32_t)rcap * tok_stride(F);
}

// The down ring: its first nb stages lie beside the gate/up ring (so they
// can be filled while gate/up still runs), the rest over the gate/up ring's
// memory, free once this block's gate/up items are done.
struct DnRing {
  uint8_t* beside;
  uint8_t* front;
  int nb;
  uint32_t sb;  // stage bytes
  __device__ __forceinline__ uint8_t* stage(int s) const {
    return s < nb ? beside + (size_t)s * sb : front + (size_t)(s - nb) * sb;
  }
};

__device__ __forceinline__ void mbar_expect_tx_only(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void issue_down_rows(const __nv_bfloat16* __restrict__ w_down, int e, int H, int F, int h0,
                                                int rows, uint32_t dst, uint32_t bar) {
  bulk_load(dst, w_down + ((int64_t)e * H + h0) * F, (uint32_t)rows * F * 2, bar);
}

// Producer lane: request the weight rows of this block's first down items
// into the ring stages beside the gate/up ring.  Returns how many.
__device__ __forceinline__ int down_prefetch(const __nv_bfloat16* __restrict__ w_down, int H, int F, int hr, int bid,
                                             int nblk, DnRing ring, uint64_t* full, Meta m) {
  DnCursor cur = dn_range(*m.nact, H, hr, bid, nblk);
  int a, h0, rows, j = 0;
  fence_proxy_async_smem();
  for (; j < ring.nb && cur.next(a, h0, rows); ++j) {
    const uint32_t bar = smem_u32(&full[j]);
    mbar_expect_tx_only(bar, (uint32_t)rows * F * 2);
    issue_down_rows(w_down, m.act[a], H, F, h0, rows, smem_u32(ring.stage(j)), bar);
  }
  return j;
}

template <class TY>
__device__ __forceinline__ void down_body(const __nv_bfloat16* __restrict__ w_down, int T, int H, int F, int E, int k,
                                          int hr, int rcap, int stages, int pre, DecodeWs ws, int bid, int nblk,
                                          DnRing ring, float* dsm, int nhmax, float* red, uint64_t* full,
                                          uint64_t* empty, int* s_abort, Meta m, TY* y) {
  const int32_t* sm_off = m.off;
  const int32_t* sm_act = m.act;
  const float* sm_w = m.w;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t hrow = (uint32_t)F * 2;  // weight row stride
  const uint32_t ts = tok_stride(F);      // h row stride
  const uint32_t stage_bytes = dn_stage_bytes(F, hr, rcap);
  const int nact = *m.nact;
  if (warp == kWarps) {
    // producer warp: refills a stage as soon as all compute warps released it
    if (lane == 0) {
      // the ring's later stages reuse the gate/up ring's memory
      fence_proxy_async_smem();
      DnCursor cur = dn_range(nact, H, hr, bid, nblk);
      int a, h0, rows;
      for (int j = 0; cur.next(a, h0, rows); ++j) {
        const int s = j % stages;
        const int e = sm_act[a];
        const uint32_t bar = smem_u32(&full[s]);
        const int r0 = sm_off[e];
        const int rc = min(rcap, sm_off[e + 1] - r0);
        const uint32_t dst = smem_u32(ring.stage(s));
        TRACE_ITEM(1, j, 2);
        if (j < pre) {  // weights already requested
          mbar_expect_tx(bar, (uint32_t)rc * hrow);
        } else {
          if (j >= stages && !mbar_wait(smem_u32(&empty[s]), (uint32_t)(j / stages - 1) & 1u, s_abort, ws.err))
            break;
          mbar_expect_tx(bar, (uint32_t)(rows + rc) * hrow);
          issue_down_rows(w_down, e, H, F, h0, rows, dst, bar);
        }
        for (int r = 0; r < rc; ++r) bulk_load(dst + hr * hrow + r * ts, ws.hs + (int64_t)(r0 + r) * F, hrow, bar);
      }
    }
    return;
  }
  DnCursor cur = dn_range(nact, H, hr, bid, nblk);
  const int hb0 = cur.hb0, nh = cur.hb1 - cur.hb0;
  int a, h0, rows, tile = 0;
  for (int j = 0; cur.next(a, h0, rows); ++j) {
    const int e = sm_act[a];
    const int s = j % stages;
    if (!mbar_wait(smem_u32(&full[s]), (uint32_t)(j / stages) & 1u, s_abort, ws.err)) break;
    if (threadIdx.x == 0) TRACE_ITEM(1, j, 0);
    uint8_t* st = ring.stage(s);
    uint8_t* hsm = st + hr * hrow;
    const int r0 = sm_off[e], cnt = sm_off[e + 1] - r0;
    for (int c0 = 0; c0 < cnt; c0 += rcap) {
      const int rc = min(rcap, cnt - c0);
      if (c0 > 0) {  // more than rcap rows: later chunks are loaded into the same area
        const int fv = F / 8;
        for (int i = threadIdx.x; i < rc * fv; i += kThreads) {
          const int r = i / fv, v = i - r * fv;
          *reinterpret_cast<uint4*>(hsm + r * ts + v * 16) =
              reinterpret_cast<const uint4*>(ws.hs + (int64_t)(r0 + c0 + r) * F)[v];
        }
        consumer_sync();
      }
      float* rb = red + (tile++ & 1) * (kWarps * kMT * 8);
      // rows 8..15 of the tile: the item's rows past 8, or (none) its own rows again
      warp_tile_mma(st, min(rows, 8), rows > 8 ? st + 8 * hrow : st, rows > 8 ? rows - 8 : rows, hrow, hsm, ts, F,
                    rc, rb);
      if (c0 + rcap >= cnt) {
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&empty[s]));  // this warp is done with stage s
      }
      consumer_sync();
      if (threadIdx.x < kMT * 8) {
        const int i = threadIdx.x >> 3, n = threadIdx.x & 7;
        if (i < rows && n < rc) {
          const int row = r0 + c0 + n;
          dsm[row * nhmax + (h0 - hb0) + i] = red_sum(rb, i, n) * sm_w[row];
        }
      }
      if (c0 + rcap < cnt) consumer_sync();  // the next chunk's rows overwrite the h area
    }
    if (threadIdx.x == 0) TRACE_ITEM(1, j, 1);
  }
  consumer_sync();  // every d value of this block is in dsm
  TRACE(6);
  // y[t, h] = sum_{j<k} d[slot j of t, h] in slot order, + residual
  for (int i = threadIdx.x; i < T * nh; i += kThreads) {
    const int t = i / nh, hh = i - t * nh;
    float acc = 0.f;
    for (int j = 0; j < k; ++j) acc += dsm[m.pos[j * T + t] * nhmax + hh];
    const int64_t o = (int64_t)t * H + hb0 + hh;
    if (ws.res) acc = ws.res[o] + acc;  // the sub-layer's residual add after the sum
    y[o] = from_f32<TY>(acc);
  }
}

template <class TY>
__global__ void __launch_bounds__(kBlockThreads)
decode_down_kernel(const __nv_bfloat16* __restrict__ w_down, int T, int H, int F, int E, int k, int hr, int rcap,
                   int stages, int nhmax, TY* y, DecodeWs ws) {
  extern __shared__ __align__(128) uint8_t dsm_raw[];
  __shared__ __align__(8) uint64_t full[8], empty[8];
  __shared__ __align__(16) float red[2 * kWarps * kMT * 8];
  __shared__ int s_abort;
  if (threadIdx.x == 0) {
    s_abort = 0;
    init_ring(full, empty, stages);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  wait_prior_grid();
  allow_next_grid();
  __shared__ int32_t m_off[kMaxE + 1], m_act[kMaxE], m_nact, m_tok[kMaxSlots], m_pos[kMaxSlots];
  __shared__ float m_w[kMaxSlots];
  const Meta m = load_meta(ws, T, E, m_off, m_act, &m_nact, m_tok, m_w, m_pos);
  const DnRing ring{dsm_raw, dsm_raw, 0, dn_stage_bytes(F, hr, rcap)};
  float* dsm = reinterpret_cast<float*>(dsm_raw + (((size_t)stages * dn_stage_bytes(F, hr, rcap) + 127) & ~(size_t)127));
  down_body<TY>(w_down, T, H, F, E, k, hr, rcap, stages, 0, ws, blockIdx.x, gridDim.x, ring, dsm, nhmax, red,
                full, empty, &s_abort, m, y);
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

// Placement of the streaming phases in the fused kernel's dynamic shared
// memory: the gate/up ring at 0; the down ring right after it when both fit
// (then the down weights of a block's first items are requested before the
// grid barrier that publishes h, overlapping the barrier and the other
// blocks' last gate/up items), else at 0 as well; the down phase's d values
// after both.  The routing phases use the start of the area before either.
struct DecodeSmem {
  size_t dn_off, dsm_off, total;
  int dn_beside;  // down stages beside the gate/up ring (requested before the barrier)
  bool prefetch;
};

template <class TW, class TY>
__global__ void __launch_bounds__(kBlockThreads, 1)
decode_fused_kernel(const __nv_bfloat16* __restrict__ x, const TW* __restrict__ wr,
                    const __nv_bfloat16* __restrict__ w_gate, const __nv_bfloat16* __restrict__ w_up,
                    const __nv_bfloat16* __restrict__ w_down, int T, int H, int F, int E, int k, int normalize,
                    int fr, int stages_gu, int hr, int stages_dn, int rcap, int nhmax, DecodeSmem lay, TY* y,
                    DecodeWs ws) {
  extern __shared__ __align__(128) uint8_t dsm_raw[];
  __shared__ __align__(8) uint64_t full_gu[4], full_dn[8], empty_gu[4], empty_dn[8];
  __shared__ __align__(16) float red[2 * kWarps * kMT * 8];
  __shared__ int s_abort;
  if (threadIdx.x == 0) {
    s_abort = 0;
    init_ring(full_gu, empty_gu, stages_gu);
    init_ring(full_dn, empty_dn, stages_dn);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  const int bid = blockIdx.x, nblk = gridDim.x;
  const bool compute = threadIdx.x < kThreads;  // warps 0..kWarps-1; the last warp produces copies
  TRACE(0);
  if (compute) route_body<TW>(x, wr, T, H, E, ws, reinterpret_cast<float*>(dsm_raw), bid, nblk);
  TRACE(1);
  grid_barrier(ws.gbar, 1u * nblk, &s_abort, ws.err);
  TRACE(2);
  // every block runs softmax / top-k for all T tokens and builds the (small)
  // permutation itself, so the streaming phases start without another
  // barrier; block 0 also publishes the routing
  __shared__ int32_t m_off[kMaxE + 1], m_act[kMaxE], m_nact, m_tok[kMaxSlots], m_pos[kMaxSlots];
  __shared__ float m_w[kMaxSlots];
  const Meta m{m_off, m_act, &m_nact, m_tok, m_w, m_pos};
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
  TRACE(3);
  gateup_body(x, w_gate, w_up, T, H, F, E, fr, rcap, stages_gu, ws, bid, nblk, dsm_raw, red, full_gu, empty_gu,
              &s_abort, m);
  TRACE(4);
  const DnRing ring{dsm_raw + lay.dn_off, dsm_raw, lay.dn_beside, dn_stage_bytes(F, hr, rcap)};
  int pre = 0;
  if (lay.prefetch && threadIdx.x == kThreads)  // the producer lane, done issuing its gate/up copies
    pre = down_prefetch(w_down, H, F, hr, bid, nblk, ring, full_dn, m);
  grid_barrier(ws.gbar, 2u * nblk, &s_abort, ws.err);
  TRACE(5);
  down_body<TY>(w_down, T, H, F, E, k, hr, rcap, stages_dn, pre, ws, bid, nblk, ring,
                reinterpret_cast<float*>(dsm_raw + lay.dsm_off), nhmax, red, full_dn, empty_dn, &s_abort, m, y);
  // every block has passed the last barrier: the last one to leave zeroes
  // both counters, so the workspace is ready for the next call
  if (threadIdx.x == 0 && atomicAdd(ws.gbar + 1, 1u) == (unsigned)nblk - 1) {
    ws.gbar[0] = 0;
    ws.gbar[1] = 0;
  }
  TRACE(7);
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

// Shared-memory staging of the two streaming phases.  An expert receives at
// most T rows (the top-k ids of a token are distinct), so a stage holds
// rcap = min(kRC, T) token rows (at a padded stride) beside its 16 weight
// rows.  Gate/up items are up to fr = 8 row pairs, down items up to
// hr = min(16, ceil(H / nblk)) rows.  A shape where two stages of either
// phase do not fit leaves the decode path.
struct DecodePlan {
  int rcap, fr, hr, stages_gu, stages_dn, nhmax;
  size_t stage_gu, stage_dn, dsm_bytes;
  DecodeSmem lay;
  bool ok;
};

// dynamic shared memory beside the kernels' static tables (< 12 KB)
constexpr size_t kSmemDyn = 227 * 1024 - 12 * 1024;

DecodePlan decode_plan(int64_t T, int64_t H, int64_t F, int64_t k, int nblk) {
  DecodePlan p{};
  p.rcap = (int)(T < kRC ? T : kRC);
  p.nhmax = (int)((H + nblk - 1) / nblk);
  p.dsm_bytes = align_up((size_t)k * T * p.nhmax * 4, 128);
  int fr_env = 0, gu_env = 0;
  if (const char* v = getenv("FRANK_DECODE_FR")) fr_env = atoi(v);
  if (const char* v = getenv("FRANK_DECODE_GU_STAGES")) gu_env = atoi(v);
  const size_t budget = kSmemDyn > p.dsm_bytes ? kSmemDyn - p.dsm_bytes : 0;
  // rows per gate/up item: 8 (one 16-row tile of gate + up rows) unless two
  // stages of that do not fit; rows per down item: the block's output rows,
  // at most 16 and at most what keeps two stages within the budget
  p.fr = 8;
  while (p.fr > 1 && 2 * (size_t)gu_stage_bytes((int)H, p.fr, p.rcap) > budget) p.fr /= 2;
  if (fr_env > 0 && fr_env < p.fr) p.fr = fr_env;
  p.hr = p.nhmax < kMT ? p.nhmax : kMT;
  while (p.hr > 1 && 2 * (size_t)dn_stage_bytes((int)F, p.hr, p.rcap) > budget) p.hr = (p.hr + 1) / 2;
  p.stage_gu = gu_stage_bytes((int)H, p.fr, p.rcap);
  p.stage_dn = dn_stage_bytes((int)F, p.hr, p.rcap);
  p.stages_gu = (int)(budget / p.stage_gu);
  // about 128 KB in flight per SM covers the loaded HBM latency
  auto depth = [](size_t stage) {
    const int want = (int)((128 * 1024 + stage - 1) / stage);
    return want < 2 ? 2 : (want > 4 ? 4 : want);
  };
  if (p.stages_gu > depth(p.stage_gu)) p.stages_gu = depth(p.stage_gu);
  if (gu_env >= 2 && gu_env <= 4 && (size_t)gu_env * p.stage_gu <= budget) p.stages_gu = gu_env;
  const size_t gu_bytes = (size_t)p.stages_gu * p.stage_gu;
  // down ring: stages beside the gate/up ring (requested before the second
  // grid barrier) and stages over the gate/up ring's memory; at most 8
  const size_t rest = budget > gu_bytes + 128 ? budget - gu_bytes - 128 : 0;
  int beside = (int)(rest / p.stage_dn);
  const char* pf = getenv("FRANK_DECODE_PREFETCH");
  if (beside < 2 || (pf && pf[0] == '0')) beside = 0;
  if (beside > 4) beside = 4;
  int front = (int)((beside ? gu_bytes : budget) / p.stage_dn);
  if (front > 8 - beside) front = 8 - beside;
  p.stages_dn = beside + front;
  p.ok = p.stages_gu >= 2 && p.stages_dn >= 2 && H % 16 == 0 && F % 16 == 0;
  p.lay.prefetch = beside > 0;
  p.lay.dn_beside = beside;
  p.lay.dn_off = beside ? align_up(gu_bytes, 128) : 0;
  const size_t dn_end = beside ? p.lay.dn_off + (size_t)beside * p.stage_dn : (size_t)front * p.stage_dn;
  const size_t ring_end = align_up(dn_end > gu_bytes ? dn_end : gu_bytes, 128);
  p.lay.dsm_off = ring_end;
  p.lay.total = ring_end + p.dsm_bytes;
  return p;
}

template <class TW, class TY>
int launch_fused(const void* x, const void* wr, const void* wg, const void* wu, const void* wd, int64_t T, int64_t H,
                 int64_t F, int64_t E, int64_t k, int normalize, const DecodePlan& pl, void* y, const DecodeWs& ws,
                 size_t smem, cudaStream_t st) {
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
                                    (int)E, (int)k, normalize, pl.fr, pl.stages_gu, pl.hr, pl.stages_dn, pl.rcap,
                                    pl.nhmax, pl.lay, (TY*)y, ws));
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

}  // namespace

namespace frank {

bool decode_path_ok(int dtype, int64_t T, int64_t H, int64_t F, int64_t E, int64_t k) {
  return dtype == FRANK_BF16 && T >= 1 && T <= 64 && k * T <= kMaxSlots && E <= kMaxE && H % 8 == 0 && F % 8 == 0 &&
         k * T <= E && decode_plan(T, H, F, k, num_sms()).ok;
}

size_t decode_workspace_size(int64_t T, int64_t H, int64_t F, int64_t E, int64_t k) {
  Carve c(nullptr, 0);
  const int64_t n = k * T;
  c.take<unsigned>(2);  // the workspace header: barrier counters (see frank_moe_ffn_block)
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
  // the first 256 bytes of a block workspace: the fused kernel's barrier and
  // exit counters, zero before the first call and left zero by every call
  ws.gbar = c.take<unsigned>(2);
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
  ws.res = residual;
  ws.n_slots = (int)n;
  ws.err = device_error_word();
  const int grid_p = num_sms();
  const DecodePlan plan = decode_plan(T, H, F, k, grid_p);
  if (!plan.ok) {
    set_error("decode block: n_embd=%lld / n_ff=%lld too large for the streaming kernels", (long long)H,
              (long long)F);
    return FRANK_EINVAL;
  }
  const char* fenv = getenv("FRANK_DECODE_FUSED");
  if (!(fenv && fenv[0] == '0')) {
    // one cooperative launch (decode_fused_kernel)
    size_t smem = plan.lay.total;
    if (fused_routing_smem(T, E) > smem) smem = fused_routing_smem(T, E);
    mark(0, st);
    int st_launch;
    if (wr_dtype == FRANK_F32 && y_dtype == FRANK_F32)
      st_launch = launch_fused<float, float>(x, wr, w_gate_p, w_up_p, w_down_p, T, H, F, E, k, normalize, plan, y, ws,
                                             smem, st);
    else if (wr_dtype == FRANK_F32)
      st_launch = launch_fused<float, __nv_bfloat16>(x, wr, w_gate_p, w_up_p, w_down_p, T, H, F, E, k, normalize,
                                                     plan, y, ws, smem, st);
    else if (y_dtype == FRANK_F32)
      st_launch = launch_fused<__nv_bfloat16, float>(x, wr, w_gate_p, w_up_p, w_down_p, T, H, F, E, k, normalize,
                                                     plan, y, ws, smem, st);
    else
      st_launch = launch_fused<__nv_bfloat16, __nv_bfloat16>(x, wr, w_gate_p, w_up_p, w_down_p, T, H, F, E, k,
                                                             normalize, plan, y, ws, smem, st);
    FRANK_TRY(st_launch);
    for (int m = 1; m <= 6; ++m) mark(m, st);
  } else {
    // the same bodies as four launches chained by programmatic dependent launch
    mark(0, st);
    const unsigned rblocks = (unsigned)grid_p;
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
    {
      const size_t smem = (size_t)plan.stages_gu * plan.stage_gu;
      FRANK_CUDA_TRY(
          cudaFuncSetAttribute(decode_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      FRANK_CUDA_TRY(launch_pdl(decode_gateup_kernel, dim3(grid_p), dim3(kBlockThreads), smem, st,
                                (const __nv_bfloat16*)x, (const __nv_bfloat16*)w_gate_p,
                                (const __nv_bfloat16*)w_up_p, (int)T, (int)H, (int)F, (int)E, plan.fr, plan.rcap,
                                plan.stages_gu, ws));
      FRANK_LAUNCH_CHECK();
    }
    mark(4, st);
    {
      const size_t smem = align_up((size_t)plan.stages_dn * plan.stage_dn, 128) + plan.dsm_bytes;
#define FRANK_DOWN_CASE(TY)                                                                                         \
  FRANK_CUDA_TRY(cudaFuncSetAttribute(decode_down_kernel<TY>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
  FRANK_CUDA_TRY(launch_pdl(decode_down_kernel<TY>, dim3(grid_p), dim3(kBlockThreads), smem, st,                      \
                            (const __nv_bfloat16*)w_down_p, (int)T, (int)H, (int)F, (int)E, (int)k, plan.hr,         \
                            plan.rcap, plan.stages_dn, plan.nhmax, (TY*)y, ws));
      if (y_dtype == FRANK_F32) {
        FRANK_DOWN_CASE(float)
      } else {
        FRANK_DOWN_CASE(__nv_bfloat16)
      }
#undef FRANK_DOWN_CASE
      FRANK_LAUNCH_CHECK();
    }
    mark(5, st);
    mark(6, st);
  }
  if (route_w) FRANK_CUDA_TRY(cudaMemcpyAsync(route_w, ws.w, n * sizeof(float), cudaMemcpyDeviceToDevice, st));
  if (route_ids)
    FRANK_CUDA_TRY(cudaMemcpyAsync(route_ids, ws.ids, n * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  return FRANK_OK;
}

}  // namespace frank

#ifdef FRANK_DECODE_TRACE
extern "C" int frank_decode_trace_read(unsigned long long* out, int nblocks) {
  return cudaMemcpyFromSymbol(out, g_decode_trace, sizeof(unsigned long long) * 8 * nblocks) == cudaSuccess ? 0 : -3;
}
extern "C" int frank_decode_items_read(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, g_decode_items, sizeof(g_decode_items)) == cudaSuccess ? 0 : -3;
}
#endif
