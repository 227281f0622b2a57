// Routing kernels: router logits + softmax + top-k (+ renorm), and the
// atomic-free stable expert permutation.
//
// Reference semantics:
//   router matmul        components/moe/moe_ffn_block.mlir:54-70, oracles/moe.py:87
//   softmax over experts moe_ffn_block.mlir:72-75, oracles/moe.py:90-91
//   top-k (ogt, desc.)   moe_ffn_block.mlir:77-89, oracles/moe.py:95-100
//   renormalisation      moe_ffn_block.mlir:91-128, oracles/moe.py:103-105
//   slot flattening      components/moe/mul_mat_id.mlir:51-53 (s = j*T + t)
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "topk.cuh"

namespace {
using namespace frank_topk;

constexpr int kRouterTok = 32;    // tokens per router block
constexpr int kRouterHc = 32;     // H chunk staged in shared memory
constexpr int kRouterThreads = 256;

template <int MaxE>
__global__ void softmax_topk_kernel(const float* __restrict__ logits, int64_t T, int E, int k,
                                    int normalize, float* __restrict__ w, int32_t* __restrict__ ids) {
  __shared__ float lg[8][MaxE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t t = (int64_t)blockIdx.x * 8 + warp;
  if (t >= T) return;
  for (int e = lane; e < E; e += 32) lg[warp][e] = logits[(int64_t)e * T + t];
  __syncwarp();
  warp_softmax_topk<MaxE>(lg[warp], E, k, normalize, w, ids, T, t);
}

// Router: a block handles kRouterTok tokens.  x and wr are staged through
// shared memory in H chunks (converted to fp32); every thread accumulates a
// few (expert, token) logits in fp32 in ascending h order.
template <class TX, class TW>
__global__ void __launch_bounds__(kRouterThreads)
router_topk_kernel(const TX* __restrict__ x, const TW* __restrict__ wr, int64_t T, int64_t H, int E,
                   int k, int normalize, float* __restrict__ w, int32_t* __restrict__ ids) {
  extern __shared__ float sm[];
  float* xs = sm;                                  // [kRouterTok][kRouterHc+1]
  float* ws = xs + kRouterTok * (kRouterHc + 1);   // [E][kRouterHc+1]
  float* lg = ws + E * (kRouterHc + 1);            // [kRouterTok][E]
  const int tid = threadIdx.x;
  const int64_t t0 = (int64_t)blockIdx.x * kRouterTok;
  const int nout = E * kRouterTok;                 // outputs of this block
  const int per = (nout + kRouterThreads - 1) / kRouterThreads;  // <= 32
  constexpr int kAcc = kMaxE * kRouterTok / kRouterThreads;
  float acc[kAcc];
#pragma unroll
  for (int i = 0; i < kAcc; ++i) acc[i] = 0.f;
  for (int64_t h0 = 0; h0 < H; h0 += kRouterHc) {
    for (int i = tid; i < kRouterTok * kRouterHc; i += kRouterThreads) {
      int r = i / kRouterHc, c = i % kRouterHc;
      int64_t t = t0 + r, h = h0 + c;
      xs[r * (kRouterHc + 1) + c] = (t < T && h < H) ? load_as_f32(x, t * H + h) : 0.f;
    }
    for (int i = tid; i < E * kRouterHc; i += kRouterThreads) {
      int r = i / kRouterHc, c = i % kRouterHc;
      int64_t h = h0 + c;
      ws[r * (kRouterHc + 1) + c] = (h < H) ? load_as_f32(wr, (int64_t)r * H + h) : 0.f;
    }
    __syncthreads();
    int hc = (H - h0) < kRouterHc ? (int)(H - h0) : kRouterHc;
#pragma unroll
    for (int i = 0; i < kAcc; ++i) {
      int o = tid + i * kRouterThreads;
      if (i < per && o < nout) {
        int tt = o % kRouterTok, e = o / kRouterTok;
        const float* xr = xs + tt * (kRouterHc + 1);
        const float* wrow = ws + e * (kRouterHc + 1);
        float a = acc[i];
        for (int c = 0; c < hc; ++c) a = fmaf(wrow[c], xr[c], a);
        acc[i] = a;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < kAcc; ++i) {
    int o = tid + i * kRouterThreads;
    if (i < per && o < nout) {
      int tt = o % kRouterTok, e = o / kRouterTok;
      lg[tt * E + e] = acc[i];
    }
  }
  __syncthreads();
  const int warp = tid >> 5;
  for (int tt = warp; tt < kRouterTok; tt += kRouterThreads / 32) {
    int64_t t = t0 + tt;
    if (t < T) warp_softmax_topk(lg + tt * E, E, k, normalize, w, ids, T, t);
  }
}

// Vector router: logits for EC experts of every token.  The block stages
// wr[e0:e0+EC, :] (fp32) in shared memory once; each warp then takes groups
// of kTPW tokens, each lane reading 8-element (16-byte for bf16) slices of
// the token rows, accumulating kTPW x EC partial dot products in registers,
// and reducing them across the warp with butterfly shuffles.  When all E
// experts fit in one pass (E <= EC) the warp goes straight on to softmax +
// top-k; otherwise logits [E, T] go to a buffer for softmax_topk_kernel.
constexpr int kTPW = 4;
constexpr int kVecThreads = 512;

template <class T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  float4 a = __ldg(reinterpret_cast<const float4*>(p));
  float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// 8 elements held as raw 16-byte words -> fp32
__device__ __forceinline__ void raw_to_f32(const uint4 (&r)[1], float (&v)[8]) {
  const uint32_t w[4] = {r[0].x, r[0].y, r[0].z, r[0].w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ void raw_to_f32(const float4 (&r)[2], float (&v)[8]) {
  v[0] = r[0].x; v[1] = r[0].y; v[2] = r[0].z; v[3] = r[0].w;
  v[4] = r[1].x; v[5] = r[1].y; v[6] = r[1].z; v[7] = r[1].w;
}

template <class TX, class TW, int EC, int S>
__global__ void __launch_bounds__(kVecThreads)
router_vec_kernel(const TX* __restrict__ x, const TW* __restrict__ wr, int64_t T, int H, int E, int k, int normalize,
                  float* __restrict__ logits, float* __restrict__ w, int32_t* __restrict__ ids) {
  // [EC][2][H / 8][4] fp32: row e's 8-column group c is split into two planes
  // (columns 8c..8c+3 in plane 0, 8c+4..8c+7 in plane 1), so that the
  // 16-byte reads of consecutive lanes fall on consecutive banks
  extern __shared__ float sw[];
  __shared__ float lg[kVecThreads / 32][kTPW][EC];
  const int e0 = blockIdx.y * EC;
  const int ec = min(EC, E - e0);
  // router rows -> shared memory, 8 elements per load, four loads in flight
  // per thread before their stores (H % 8 == 0 on this path).  Every block
  // reads the same rows: each starts at its own 128-byte-aligned rotation so
  // that the blocks do not all ask the same L2 lines at the same time.
  const int nv = EC * H / 8;
  int rot = (int)(((int64_t)blockIdx.x * nv) / gridDim.x) & ~3;
  if (rot >= nv) rot = 0;
  for (int j0 = threadIdx.x; j0 < nv; j0 += 4 * kVecThreads) {
    float v[4][8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      int i = j0 + q * kVecThreads + rot;
      if (i >= nv) i -= nv;
      const int e = i * 8 / H, h = i * 8 - e * H;
      if (j0 + q * kVecThreads < nv && e < ec) load8(wr + (int64_t)(e0 + e) * H + h, v[q]);
      else
#pragma unroll
        for (int j = 0; j < 8; ++j) v[q][j] = 0.f;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      int i = j0 + q * kVecThreads + rot;
      if (i >= nv) i -= nv;
      if (j0 + q * kVecThreads < nv) {
        const int e = i * 8 / H, c = i - e * (H / 8);
        float4* d = reinterpret_cast<float4*>(sw + (size_t)e * H) + c;
        d[0] = make_float4(v[q][0], v[q][1], v[q][2], v[q][3]);
        d[H / 8] = make_float4(v[q][4], v[q][5], v[q][6], v[q][7]);
      }
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The block's warps are S column slices x (16 / S) token groups: with few
  // tokens the H dimension is split so that every SM has work.  Slice s of
  // warp w is w % S; its columns [hs, he) are 8-aligned.
  constexpr int kWarps = kVecThreads / 32;
  const int gpb = kWarps / S;  // token groups per block step
  const int s = warp % S, gi = warp / S;
  const int hs = (int)(((int64_t)s * (H / 8)) / S) * 8, he = (int)(((int64_t)(s + 1) * (H / 8)) / S) * 8;
  const int64_t groups = (T + kTPW - 1) / kTPW;
  const int64_t units = (groups + gpb - 1) / gpb;
  const bool fused = (E <= EC);
  // the unit loop is uniform over the block (its bound depends on blockIdx
  // only), so the block barriers of the slice reduction are reached by all
  for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
    const int64_t g = u * gpb + gi;
    const int64_t t0 = g * kTPW;
    float acc[kTPW][EC];
#pragma unroll
    for (int a = 0; a < kTPW; ++a)
#pragma unroll
      for (int e = 0; e < EC; ++e) acc[a][e] = 0.f;
    // the token loads of the next 256-column step are in flight while this
    // step's products are summed (two steps of x per warp outstanding)
    using RawX = typename std::conditional<sizeof(TX) == 2, uint4, float4>::type;
    constexpr int kRaw = sizeof(TX) == 2 ? 1 : 2;  // 16-byte words per 8 elements
    RawX xn[kTPW][kRaw];
#pragma unroll
    for (int a = 0; a < kTPW; ++a)
#pragma unroll
      for (int q = 0; q < kRaw; ++q)
        xn[a][q] = (hs + lane * 8 < he && t0 + a < T)
                       ? __ldg(reinterpret_cast<const RawX*>(x + (t0 + a) * H + hs + lane * 8) + q)
                       : RawX{};
    for (int h = hs + lane * 8; t0 < T && h < he; h += 256) {
      float xv[kTPW][8];
#pragma unroll
      for (int a = 0; a < kTPW; ++a) raw_to_f32(xn[a], xv[a]);
#pragma unroll
      for (int a = 0; a < kTPW; ++a)
#pragma unroll
        for (int q = 0; q < kRaw; ++q)
          xn[a][q] = (h + 256 < he && t0 + a < T)
                         ? __ldg(reinterpret_cast<const RawX*>(x + (t0 + a) * H + h + 256) + q)
                         : RawX{};
#pragma unroll
      for (int e = 0; e < EC; ++e) {
        const float4* we = reinterpret_cast<const float4*>(sw + e * H) + h / 8;
        const float4 w0 = we[0];
        const float4 w1 = we[H / 8];
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int a = 0; a < kTPW; ++a)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[a][e] = fmaf(wv[i], xv[a][i], acc[a][e]);
      }
    }
#pragma unroll
    for (int a = 0; a < kTPW; ++a)
#pragma unroll
      for (int e = 0; e < EC; ++e) {
        float v = acc[a][e];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[a][e] = v;
      }
    // warp sums -> shared memory; with S > 1 slice 0 adds the slices'
    // partials in slice order, one (token, expert) entry per lane
    if (lane == 0)
#pragma unroll
      for (int a = 0; a < kTPW; ++a)
#pragma unroll
        for (int e = 0; e < EC; ++e) lg[warp][a][e] = acc[a][e];
    if (S > 1) {
      __syncthreads();
      if (s == 0)
        for (int l = lane; l < kTPW * EC; l += 32) {
          float v = lg[warp][l / EC][l % EC];
          for (int s2 = 1; s2 < S; ++s2) v += lg[warp + s2][l / EC][l % EC];
          lg[warp][l / EC][l % EC] = v;
        }
      __syncthreads();
      // the block's gpb x kTPW tokens are spread over all its warps
      for (int j = warp; j < gpb * kTPW; j += kWarps) {
        const int gj = j / kTPW, a = j - gj * kTPW;
        const int64_t t = (u * gpb + gj) * kTPW + a;
        if (t >= T) continue;
        if (fused) {
          warp_softmax_topk<32>(lg[gj * S][a], E, k, normalize, w, ids, T, t);
        } else {
          for (int e = lane; e < ec; e += 32) logits[(int64_t)(e0 + e) * T + t] = lg[gj * S][a][e];
        }
      }
    } else if (t0 < T) {
      __syncwarp();
      if (fused) {
        for (int a = 0; a < kTPW; ++a)
          if (t0 + a < T) warp_softmax_topk<32>(lg[warp][a], E, k, normalize, w, ids, T, t0 + a);
      } else if (lane < kTPW && t0 + lane < T) {
#pragma unroll
        for (int e = 0; e < EC; ++e)
          if (e < ec) logits[(int64_t)(e0 + e) * T + t0 + lane] = lg[warp][lane][e];
      }
    }
    if (S > 1) __syncthreads();  // lg is rewritten by the next unit
    else __syncwarp();
  }
}

// Tensor-core router for many experts.  wr (fp32) is split exactly into three
// bf16 terms, hi = bf16(w), mid = bf16(w - hi), lo = bf16(w - hi - mid)
// (hi + mid + lo carries all 24 bits of w), stacked as a [3E, H] matrix, so
// logits = x.hi + x.mid + x.lo comes out of one bf16 GEMM with fp32
// accumulation (x is bf16, hence exact in the products).  The three partial
// dot products are added in fp32 before softmax + top-k.
template <class TW>
__global__ void router_split_kernel(const TW* __restrict__ wr, int E, int H, __nv_bfloat16* __restrict__ wr3,
                                    float* __restrict__ wr32) {
  const int64_t EH = (int64_t)E * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < EH; i += (int64_t)gridDim.x * blockDim.x) {
    const float w = load_as_f32(wr, i);
    if (wr32 != nullptr) wr32[i] = w;
    const __nv_bfloat16 hi = __float2bfloat16_rn(w);
    const float r1 = w - __bfloat162float(hi);
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    const __nv_bfloat16 lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
    wr3[i] = hi;
    wr3[EH + i] = mid;
    wr3[2 * EH + i] = lo;
  }
}

// One warp per token: logits[e] = (p[e] + p[E+e]) + p[2E+e] from the [T, 3E]
// GEMM output, then softmax + top-k.
template <int MaxE>
__global__ void softmax_topk3_kernel(const float* __restrict__ l3, int64_t T, int E, int k, int normalize,
                                     float* __restrict__ w, int32_t* __restrict__ ids) {
  __shared__ float lg[8][MaxE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * 8 + warp;
  if (t >= T) return;
  const float* row = l3 + t * 3 * E;
  for (int e = lane; e < E; e += 32) lg[warp][e] = (row[e] + row[E + e]) + row[2 * E + e];
  __syncwarp();
  warp_softmax_topk<MaxE>(lg[warp], E, k, normalize, w, ids, T, t);
}

// ---------------------------------------------------------------- permute --
// Three passes, no atomics:
//  A) per chunk of kChunk slots: stable local rank of each slot among the
//     chunk's slots of the same expert, and the chunk's per-expert counts;
//  B) one block: per-(chunk, expert) base rows and the expert offsets;
//  C) scatter: pos = base[chunk][e] + local_rank.
constexpr int kPermThreads = 256;
constexpr int kChunk = 1024;
constexpr int kPermMaxE = 1024;

__global__ void __launch_bounds__(kPermThreads)
permute_rank_kernel(const int32_t* __restrict__ ids, int64_t n, int E, int32_t* __restrict__ local_rank,
                    int32_t* __restrict__ chunk_counts, int32_t* __restrict__ err) {
  __shared__ int32_t running[kPermMaxE];
  __shared__ int32_t warp_cnt[kPermThreads / 32][kPermMaxE];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < E; e += kPermThreads) {
    running[e] = 0;
    for (int w = 0; w < kPermThreads / 32; ++w) warp_cnt[w][e] = 0;
  }
  __syncthreads();
  const int64_t c0 = (int64_t)blockIdx.x * kChunk;
  for (int base = 0; base < kChunk; base += kPermThreads) {
    int64_t s = c0 + base + tid;
    int e = -1;
    if (s < n) {
      e = ids[s];
      if (e < 0 || e >= E) {
        if (err) *err = 1;
        e = e < 0 ? 0 : E - 1;
      }
    }
    unsigned peers = __match_any_sync(0xffffffffu, e);
    int rank_w = __popc(peers & ((1u << lane) - 1u));
    int leader = __ffs(peers) - 1;
    if (e >= 0 && lane == leader) warp_cnt[warp][e] = __popc(peers);
    __syncthreads();
    int pos = 0;
    bool last = false;
    if (e >= 0) {
      int before = 0;
      for (int w = 0; w < warp; ++w) before += warp_cnt[w][e];
      pos = running[e] + before + rank_w;
      local_rank[s] = pos;
      bool last_in_warp = (lane == 31 - __clz(peers));
      last = last_in_warp;
      for (int w = warp + 1; w < kPermThreads / 32 && last; ++w)
        if (warp_cnt[w][e] != 0) last = false;
    }
    __syncthreads();
    if (last) running[e] = pos + 1;
    if (e >= 0 && lane == leader) warp_cnt[warp][e] = 0;
    __syncthreads();
  }
  for (int e = tid; e < E; e += kPermThreads) chunk_counts[(int64_t)blockIdx.x * E + e] = running[e];
}

// chunk_counts[nc][E] -> chunk_base[nc][E] (absolute rows), offsets[E+1].
__global__ void __launch_bounds__(1024)
permute_scan_kernel(const int32_t* __restrict__ chunk_counts, int nc, int E,
                    int32_t* __restrict__ chunk_base, int32_t* __restrict__ offsets) {
  __shared__ int32_t tot[kPermMaxE];
  __shared__ int32_t warp_sums[32];
  const int e = threadIdx.x;
  int32_t run = 0;
  if (e < E) {
    for (int c = 0; c < nc; ++c) {
      chunk_base[(int64_t)c * E + e] = run;
      run += chunk_counts[(int64_t)c * E + e];
    }
  }
  tot[e] = (e < E) ? run : 0;
  __syncthreads();
  // exclusive scan of tot over the block (1024 threads)
  const int lane = e & 31, warp = e >> 5;
  int v = tot[e];
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int ws = warp_sums[lane];
    int wi = ws;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += u;
    }
    warp_sums[lane] = wi - ws;
  }
  __syncthreads();
  int excl = warp_sums[warp] + incl - v;
  if (e < E) {
    offsets[e] = excl;
    if (e == E - 1) offsets[E] = excl + v;
    for (int c = 0; c < nc; ++c) chunk_base[(int64_t)c * E + e] += excl;
  }
}

__global__ void permute_scatter_kernel(const int32_t* __restrict__ ids, int64_t n, int E,
                                       const int32_t* __restrict__ local_rank,
                                       const int32_t* __restrict__ chunk_base,
                                       int32_t* __restrict__ sorted_slots,
                                       int32_t* __restrict__ slot_pos) {
  int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= n) return;
  int e = ids[s];
  e = e < 0 ? 0 : (e >= E ? E - 1 : e);
  int64_t c = s / kChunk;
  int32_t pos = chunk_base[c * E + e] + local_rank[s];
  sorted_slots[pos] = (int32_t)s;
  if (slot_pos) slot_pos[s] = pos;
}

// Small batches (n <= kSmallRounds * 1024 slots, E <= kSmallMaxE): the whole
// permutation in one block.  Round r takes slots [1024 r, 1024 r + 1024),
// one per thread; a slot's rank among the same expert's slots is the
// expert's running count before the round + the same-expert slots of lower
// warps + those of lower lanes (warp match), which is the stable order.  The
// expert totals are then scanned in the block and every thread scatters the
// slots it kept in registers (and, if asked, their gate weights into expert-
// sorted order).  Same results as the three-pass form.
constexpr int kSmallThreads = 1024;
constexpr int kSmallRounds = 4;  // past 4096 slots the three passes are as fast (measured at 8192)
constexpr int kSmallMaxE = 256;

__global__ void __launch_bounds__(kSmallThreads)
permute_small_kernel(const int32_t* __restrict__ ids, int n, int E, int32_t* __restrict__ sorted_slots,
                     int32_t* __restrict__ offsets, int32_t* __restrict__ slot_pos, int32_t* __restrict__ err,
                     const float* __restrict__ w, float* __restrict__ w_sorted) {
  constexpr int kWarps = kSmallThreads / 32;
  __shared__ int32_t running[kSmallMaxE];
  __shared__ int32_t warp_cnt[kWarps][kSmallMaxE];
  __shared__ int32_t warp_sums[kWarps];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < E; e += kSmallThreads) running[e] = 0;
  for (int i = tid; i < kWarps * kSmallMaxE; i += kSmallThreads) (&warp_cnt[0][0])[i] = 0;
  __syncthreads();
  int my_e[kSmallRounds], my_rank[kSmallRounds];
#pragma unroll
  for (int r = 0; r < kSmallRounds; ++r) {
    my_e[r] = -1;
    my_rank[r] = 0;
    if (r * kSmallThreads >= n) continue;  // uniform over the block
    const int s = r * kSmallThreads + tid;
    int e = -1;
    if (s < n) {
      e = ids[s];
      if (e < 0 || e >= E) {
        if (err) *err = 1;
        e = e < 0 ? 0 : E - 1;
      }
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int leader = __ffs(peers) - 1;
    if (e >= 0 && lane == leader) warp_cnt[warp][e] = __popc(peers);
    __syncthreads();
    bool last = false;
    if (e >= 0) {
      int before = running[e];
      for (int w = 0; w < warp; ++w) before += warp_cnt[w][e];
      my_rank[r] = before + __popc(peers & ((1u << lane) - 1u));
      my_e[r] = e;
      // the expert's last slot of the round advances its running count
      last = (lane == 31 - __clz(peers));
      for (int w = warp + 1; w < kWarps && last; ++w)
        if (warp_cnt[w][e] != 0) last = false;
    }
    __syncthreads();
    if (last) running[e] = my_rank[r] + 1;
    if (e >= 0 && lane == leader) warp_cnt[warp][e] = 0;
    __syncthreads();
  }
  // exclusive scan of the expert totals (E <= kSmallMaxE <= kSmallThreads)
  const int v = tid < E ? running[tid] : 0;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int ws = warp_sums[lane];
    int wi = ws;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += u;
    }
    warp_sums[lane] = wi - ws;
  }
  __syncthreads();
  const int excl = warp_sums[warp] + incl - v;
  __syncthreads();  // everyone has read running[] before it becomes the offsets
  if (tid < E) {
    running[tid] = excl;
    offsets[tid] = excl;
    if (tid == E - 1) offsets[E] = excl + v;
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < kSmallRounds; ++r) {
    if (my_e[r] < 0) continue;
    const int s = r * kSmallThreads + tid;
    const int32_t pos = running[my_e[r]] + my_rank[r];
    sorted_slots[pos] = s;
    if (slot_pos) slot_pos[s] = pos;
    if (w_sorted) w_sorted[pos] = w[s];
  }
}

}  // namespace

namespace frank {

int launch_softmax_topk(const float* logits, int64_t T, int64_t E, int64_t k, int normalize,
                        float* w, int32_t* ids, cudaStream_t st) {
  if (T == 0) return FRANK_OK;
  // the per-lane arrays are sized by the next multiple of 32 >= E (32..256)
#define FRANK_SOFTMAX_LAUNCH(MAXE) \
  softmax_topk_kernel<MAXE><<<(unsigned)((T + 7) / 8), 256, 0, st>>>(logits, T, (int)E, (int)k, normalize, w, ids)
  if (E <= 32) FRANK_SOFTMAX_LAUNCH(32);
  else if (E <= 64) FRANK_SOFTMAX_LAUNCH(64);
  else if (E <= 128) FRANK_SOFTMAX_LAUNCH(128);
  else FRANK_SOFTMAX_LAUNCH(kMaxE);
#undef FRANK_SOFTMAX_LAUNCH
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

static int launch_router_legacy(int x_dtype, const void* x, int wr_dtype, const void* wr, int64_t T, int64_t H,
                                int64_t E, int64_t k, int normalize, float* w, int32_t* ids, cudaStream_t st) {
  size_t smem = sizeof(float) * (kRouterTok * (kRouterHc + 1) + E * (kRouterHc + 1) + kRouterTok * E);
  dim3 grid((unsigned)((T + kRouterTok - 1) / kRouterTok));
#define FRANK_ROUTER_CASE(TX, TW)                                                                 \
  {                                                                                               \
    auto kern = router_topk_kernel<TX, TW>;                                                       \
    FRANK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    kern<<<grid, kRouterThreads, smem, st>>>((const TX*)x, (const TW*)wr, T, H, (int)E, (int)k,   \
                                             normalize, w, ids);                                  \
  }
  if (x_dtype == FRANK_F32 && wr_dtype == FRANK_F32) FRANK_ROUTER_CASE(float, float)
  else if (x_dtype == FRANK_F32) FRANK_ROUTER_CASE(float, __nv_bfloat16)
  else if (wr_dtype == FRANK_F32) FRANK_ROUTER_CASE(__nv_bfloat16, float)
  else FRANK_ROUTER_CASE(__nv_bfloat16, __nv_bfloat16)
#undef FRANK_ROUTER_CASE
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

template <class TX, class TW, int EC, int S>
static int launch_router_vec_s(const void* x, const void* wr, int64_t T, int64_t H, int64_t E, int64_t k,
                               int normalize, float* logits, float* w, int32_t* ids, cudaStream_t st) {
  auto kern = router_vec_kernel<TX, TW, EC, S>;
  const size_t smem = (size_t)EC * H * sizeof(float);
  // attribute and occupancy are fixed per kernel, device and size: queried
  // once per device (and again when a larger H needs more shared memory)
  constexpr int kDevs = 64;
  static std::mutex mu;
  static size_t set_smem[kDevs] = {};
  static int occ[kDevs] = {};
  int dev = 0;
  FRANK_CUDA_TRY(cudaGetDevice(&dev));
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= kDevs || set_smem[dev] < smem) {
      FRANK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      FRANK_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kVecThreads, smem));
      if (dev < kDevs) {
        set_smem[dev] = smem;
        occ[dev] = per_sm;
      }
    } else {
      per_sm = occ[dev];
    }
  }
  const int64_t passes = (E + EC - 1) / EC;
  const int64_t groups = (T + kTPW - 1) / kTPW;
  const int64_t gpb = (kVecThreads / 32) / S;
  int64_t gx = (groups + gpb - 1) / gpb;
  int64_t cap = (int64_t)num_sms() * (per_sm > 0 ? per_sm : 1);
  cap = (cap + passes - 1) / passes;
  if (gx > cap) gx = cap;
  dim3 grid((unsigned)(gx < 1 ? 1 : gx), (unsigned)passes);
  kern<<<grid, kVecThreads, smem, st>>>((const TX*)x, (const TW*)wr, T, (int)H, (int)E, (int)k, normalize, logits, w,
                                        ids);
  FRANK_LAUNCH_CHECK();
  if (passes > 1) FRANK_TRY(launch_softmax_topk(logits, T, E, k, normalize, w, ids, st));
  return FRANK_OK;
}

// H is split over S warps of a block when the token groups alone fill fewer
// than one block per SM for each pass over the experts.
template <class TX, class TW, int EC>
static int launch_router_vec_t(const void* x, const void* wr, int64_t T, int64_t H, int64_t E, int64_t k,
                               int normalize, float* logits, float* w, int32_t* ids, cudaStream_t st) {
  const int64_t passes = (E + EC - 1) / EC;
  const int64_t groups = (T + kTPW - 1) / kTPW;
  const int64_t want = ((int64_t)num_sms() + passes - 1) / passes;  // blocks per pass
  int S = 1;
  while (S < 8 && groups * S < want * (kVecThreads / 32) && H / 8 >= 32 * 2 * S) S *= 2;  // each slice keeps >= 32 lanes x 8 columns
  switch (S) {
    case 1: return launch_router_vec_s<TX, TW, EC, 1>(x, wr, T, H, E, k, normalize, logits, w, ids, st);
    case 2: return launch_router_vec_s<TX, TW, EC, 2>(x, wr, T, H, E, k, normalize, logits, w, ids, st);
    case 4: return launch_router_vec_s<TX, TW, EC, 4>(x, wr, T, H, E, k, normalize, logits, w, ids, st);
    default: return launch_router_vec_s<TX, TW, EC, 8>(x, wr, T, H, E, k, normalize, logits, w, ids, st);
  }
}

template <class TX, class TW>
static int launch_router_vec(const void* x, const void* wr, int64_t T, int64_t H, int64_t E, int64_t k, int normalize,
                             float* logits, float* w, int32_t* ids, cudaStream_t st) {
  const int64_t budget = 160 * 1024;
  if (8 * H * 4 <= budget) return launch_router_vec_t<TX, TW, 8>(x, wr, T, H, E, k, normalize, logits, w, ids, st);
  if (4 * H * 4 <= budget) return launch_router_vec_t<TX, TW, 4>(x, wr, T, H, E, k, normalize, logits, w, ids, st);
  if (2 * H * 4 <= budget) return launch_router_vec_t<TX, TW, 2>(x, wr, T, H, E, k, normalize, logits, w, ids, st);
  return launch_router_vec_t<TX, TW, 1>(x, wr, T, H, E, k, normalize, logits, w, ids, st);
}

int launch_tc_grouped_gemm(int, const void*, const void*, const void*, const int32_t*, int64_t, int64_t, int64_t,
                           int64_t, const float*, void*, cudaStream_t, const int32_t*, const int32_t*, float* const*,
                           int, int64_t);

static bool router_tc_ok(int x_dtype, int64_t T, int64_t H, int64_t E) {
  return x_dtype == FRANK_BF16 && E >= 16 && E % 16 == 0 && E <= kMaxE && H % 8 == 0 && T >= 128;
}

size_t router_scratch_bytes(int x_dtype, int64_t T, int64_t H, int64_t E) {
  if (router_tc_ok(x_dtype, T, H, E))
    return align_up((size_t)T * 3 * E * 4, 256) + align_up((size_t)3 * E * H * 2, 256) + 256;
  return E <= 8 ? 0 : (size_t)T * E * sizeof(float);
}

static int launch_router_split(int wr_dtype, const void* wr, int64_t E, int64_t H, __nv_bfloat16* wr3, float* wr32,
                               cudaStream_t st) {
  const int64_t EH = E * H;
  const unsigned blocks = (unsigned)((EH + 255) / 256 < 1024 ? (EH + 255) / 256 : 1024);
  if (wr_dtype == FRANK_F32)
    router_split_kernel<float><<<blocks, 256, 0, st>>>((const float*)wr, (int)E, (int)H, wr3, wr32);
  else
    router_split_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>((const __nv_bfloat16*)wr, (int)E, (int)H, wr3, wr32);
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

size_t router_pack_offset(int64_t E, int64_t H) { return align_up((size_t)E * H * 4, 256); }
size_t router_pack_bytes(int64_t E, int64_t H) { return router_pack_offset(E, H) + align_up((size_t)3 * E * H * 2, 256); }

int launch_router_pack(int wr_dtype, const void* wr, int64_t E, int64_t H, void* pack, cudaStream_t st) {
  char* base = static_cast<char*>(pack);
  return launch_router_split(wr_dtype, wr, E, H, reinterpret_cast<__nv_bfloat16*>(base + router_pack_offset(E, H)),
                             reinterpret_cast<float*>(base), st);
}

// wr3_pre: the prepared split of a router pack (or null: split wr here).
static int launch_router_tc(const void* x, int wr_dtype, const void* wr, const __nv_bfloat16* wr3_pre, int64_t T,
                            int64_t H, int64_t E, int64_t k, int normalize, float* w, int32_t* ids, void* scratch,
                            cudaStream_t st) {
  Carve c(scratch, router_scratch_bytes(FRANK_BF16, T, H, E));
  float* l3 = c.take<float>(T * 3 * E);
  __nv_bfloat16* wr3 = c.take<__nv_bfloat16>(3 * E * H);
  if (wr3_pre == nullptr) FRANK_TRY(launch_router_split(wr_dtype, wr, E, H, wr3, nullptr, st));
  // one group of T rows: no offsets array needed
  FRANK_TRY(launch_tc_grouped_gemm(2, x, wr3_pre ? wr3_pre : wr3, nullptr, nullptr, 1, T, 3 * E, H, nullptr, l3, st,
                                   nullptr, nullptr, nullptr, 0, 0));
#define FRANK_SOFTMAX3_LAUNCH(MAXE) \
  softmax_topk3_kernel<MAXE><<<(unsigned)((T + 7) / 8), 256, 0, st>>>(l3, T, (int)E, (int)k, normalize, w, ids)
  if (E <= 32) FRANK_SOFTMAX3_LAUNCH(32);
  else if (E <= 64) FRANK_SOFTMAX3_LAUNCH(64);
  else if (E <= 128) FRANK_SOFTMAX3_LAUNCH(128);
  else FRANK_SOFTMAX3_LAUNCH(kMaxE);
#undef FRANK_SOFTMAX3_LAUNCH
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

// logits: scratch of router_scratch_bytes(x_dtype, T, H, E) bytes (may be null: slower kernels).
int launch_router_topk(int x_dtype, const void* x, int wr_dtype, const void* wr, int64_t T, int64_t H,
                       int64_t E, int64_t k, int normalize, float* w, int32_t* ids, float* logits, cudaStream_t st,
                       const __nv_bfloat16* wr3_pre) {
  if (T == 0) return FRANK_OK;
  if (logits != nullptr && router_tc_ok(x_dtype, T, H, E) && (uintptr_t)x % 16 == 0)
    return launch_router_tc(x, wr_dtype, wr, wr3_pre, T, H, E, k, normalize, w, ids, logits, st);
  const size_t esz = x_dtype == FRANK_F32 ? 4 : 2;
  const bool vec_ok = (H % 8 == 0) && ((uintptr_t)x % 16 == 0) && ((uintptr_t)wr % 16 == 0) &&
                      (H * 4 * 1 <= 160 * 1024) &&
                      (E <= 8 || logits != nullptr) && (H * esz) % 16 == 0;
  if (!vec_ok) return launch_router_legacy(x_dtype, x, wr_dtype, wr, T, H, E, k, normalize, w, ids, st);
  if (x_dtype == FRANK_F32 && wr_dtype == FRANK_F32)
    return launch_router_vec<float, float>(x, wr, T, H, E, k, normalize, logits, w, ids, st);
  if (x_dtype == FRANK_F32)
    return launch_router_vec<float, __nv_bfloat16>(x, wr, T, H, E, k, normalize, logits, w, ids, st);
  if (wr_dtype == FRANK_F32)
    return launch_router_vec<__nv_bfloat16, float>(x, wr, T, H, E, k, normalize, logits, w, ids, st);
  return launch_router_vec<__nv_bfloat16, __nv_bfloat16>(x, wr, T, H, E, k, normalize, logits, w, ids, st);
}

size_t permute_workspace_size(int64_t n, int64_t E) {
  int64_t nc = (n + kChunk - 1) / kChunk;
  return align_up(n * 4, 256) + 2 * align_up(nc * E * 4, 256) + 256;
}

int launch_sorted_weights(const float*, const int32_t*, int64_t, float*, cudaStream_t);

// w / w_sorted (both or neither): also w_sorted[r] = w[sorted_slots[r]].
int launch_permute(const int32_t* ids, int64_t n, int64_t E, int32_t* sorted_slots, int32_t* offsets,
                   int32_t* slot_pos, int32_t* err, void* ws, size_t ws_bytes, cudaStream_t st, const float* w,
                   float* w_sorted) {
  if (E < 1 || E > kPermMaxE) {
    set_error("permute: E=%lld outside [1, %d]", (long long)E, kPermMaxE);
    return FRANK_EINVAL;
  }
  if (ws_bytes < permute_workspace_size(n, E)) {
    set_error("permute: workspace %zu < %zu bytes", ws_bytes, permute_workspace_size(n, E));
    return FRANK_ENOSPC;
  }
  if (n == 0) {
    FRANK_CUDA_TRY(cudaMemsetAsync(offsets, 0, (E + 1) * sizeof(int32_t), st));
    return FRANK_OK;
  }
  if (n <= (int64_t)kSmallRounds * kSmallThreads && E <= kSmallMaxE) {
    permute_small_kernel<<<1, kSmallThreads, 0, st>>>(ids, (int)n, (int)E, sorted_slots, offsets, slot_pos, err,
                                                      w, w_sorted);
    FRANK_LAUNCH_CHECK();
    return FRANK_OK;
  }
  int64_t nc = (n + kChunk - 1) / kChunk;
  Carve c(ws, ws_bytes);
  int32_t* local_rank = c.take<int32_t>(n);
  int32_t* counts = c.take<int32_t>(nc * E);
  int32_t* base = c.take<int32_t>(nc * E);
  permute_rank_kernel<<<(unsigned)nc, kPermThreads, 0, st>>>(ids, n, (int)E, local_rank, counts, err);
  FRANK_LAUNCH_CHECK();
  permute_scan_kernel<<<1, 1024, 0, st>>>(counts, (int)nc, (int)E, base, offsets);
  FRANK_LAUNCH_CHECK();
  permute_scatter_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(ids, n, (int)E, local_rank, base,
                                                                       sorted_slots, slot_pos);
  FRANK_LAUNCH_CHECK();
  if (w_sorted) return launch_sorted_weights(w, sorted_slots, n, w_sorted, st);
  return FRANK_OK;
}

}  // namespace frank
