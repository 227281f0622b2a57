// Decode-sized MoE FFN block (a few tokens per step): four launches,
// weight-streaming on CUDA cores.
//
// With T <= 64 tokens an expert receives a handful of rows, so the block is
// bound by reading the active experts' weights from HBM (3 x H x F bf16 per
// active expert) -- tensor cores would idle on 128-row tiles.  The kernels:
//   decode_route_kernel    router logits (one warp per (expert, 8 tokens));
//                          the last block to finish runs softmax + top-k +
//                          renorm for every token, the stable expert
//                          permutation and the list of active experts
//                          (moe_ffn_block.mlir:54-128, mul_mat_id.mlir:51-53);
//   decode_gateup_kernel   persistent blocks over (active expert, 8 rows of F):
//                          one gate row and one up row per warp streamed once
//                          and dotted with the expert's token rows (gathered
//                          straight from x), h = gate * silu(up)
//                          (swiglu.mlir:37-47);
//   decode_down_kernel     persistent blocks over (active expert, 32 rows of
//                          H): d = down(h) * gate weight, fp32;
//   combine_kernel         y[t] = sum of the k slots of t in slot order
//                          (moe_ffn_block.mlir:179-206), deterministic.
// The only atomic is the completion ticket of the route kernel; it resets
// itself, and the launcher zeroes it at every call.
#include "common.cuh"
#include "topk.cuh"

namespace {

using namespace frank_topk;

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRouteTok = 8;    // tokens per route warp item
constexpr int kMaxSlots = 2048; // k * T handled by the decode path
constexpr int kRC = 8;          // token rows per pass over an expert's weights

__device__ __forceinline__ void bf16x8_to_f32(uint4 u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// Same as bf16x8_to_f32, but opaque to the optimiser so that the unpacking
// stays next to its use (it must not be hoisted out of the per-row loops,
// which would keep 64+ unpacked floats live per lane).
__device__ __forceinline__ void bf16x8_unpack_here(uint4 u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t lo, hi;
    asm volatile("shl.b32 %0, %2, 16;\n\tand.b32 %1, %2, 0xffff0000;" : "=r"(lo), "=r"(hi) : "r"(w[i]));
    v[2 * i] = __uint_as_float(lo);
    v[2 * i + 1] = __uint_as_float(hi);
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
  unsigned* ticket;     // completion counter of the route kernel
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
};

// ----------------------------------------------------------------- route --
template <class TW>
__global__ void __launch_bounds__(kThreads)
decode_route_kernel(const __nv_bfloat16* __restrict__ x, const TW* __restrict__ wr, int T, int H, int E, int k,
                    int normalize, DecodeWs ws) {
  asm volatile("griddepcontrol.launch_dependents;" :::);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tchunks = (T + kRouteTok - 1) / kRouteTok;
  const int item = blockIdx.x * kWarps + warp;
  if (item < E * tchunks) {
    const int e = item / tchunks, t0 = (item - e * tchunks) * kRouteTok;
    float acc[kRouteTok];
#pragma unroll
    for (int a = 0; a < kRouteTok; ++a) acc[a] = 0.f;
#pragma unroll 8
    for (int h = lane * 8; h < H; h += 256) {
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
#pragma unroll
    for (int a = 0; a < kRouteTok; ++a) {
      float v = acc[a];
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && t0 + a < T) ws.logits[(int64_t)e * T + t0 + a] = v;
    }
  }
  // ---- the last block: softmax + top-k for every token, then the permutation
  __shared__ unsigned s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(ws.ticket, 1u) == gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  __shared__ float lg[kWarps][kMaxE];
  for (int t = warp; t < T; t += kWarps) {
    for (int e = lane; e < E; e += 32) lg[warp][e] = ws.logits[(int64_t)e * T + t];
    __syncwarp();
    warp_softmax_topk(lg[warp], E, k, normalize, ws.w, ws.ids, T, t);
    __syncwarp();
  }
  __syncthreads();
  // stable counting sort of the n = k*T flat slots by expert (same order as
  // argsort(ids.reshape(-1), stable)); one block, warp-level ranks
  __shared__ int32_t running[kMaxE + 1];
  __shared__ int32_t warp_cnt[kWarps][kMaxE];
  __shared__ int32_t rank[kMaxSlots];
  const int n = k * T;
  for (int e = threadIdx.x; e < E; e += kThreads) {
    running[e] = 0;
    for (int w2 = 0; w2 < kWarps; ++w2) warp_cnt[w2][e] = 0;
  }
  __syncthreads();
  for (int base = 0; base < n; base += kThreads) {
    const int s = base + threadIdx.x;
    const int e = s < n ? ws.ids[s] : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_w = __popc(peers & ((1u << lane) - 1u));
    const int leader = __ffs(peers) - 1;
    if (e >= 0 && lane == leader) warp_cnt[warp][e] = __popc(peers);
    __syncthreads();
    int pos = 0;
    bool last = false;
    if (e >= 0) {
      int before = 0;
      for (int w2 = 0; w2 < warp; ++w2) before += warp_cnt[w2][e];
      pos = running[e] + before + rank_w;
      rank[s] = pos;
      last = (lane == 31 - __clz(peers));
      for (int w2 = warp + 1; w2 < kWarps && last; ++w2)
        if (warp_cnt[w2][e] != 0) last = false;
    }
    __syncthreads();
    if (last) running[e] = pos + 1;
    if (e >= 0 && lane == leader) warp_cnt[warp][e] = 0;
    __syncthreads();
  }
  if (threadIdx.x == 0) {  // exclusive scan of the counts (E <= 256)
    int32_t acc = 0;
    for (int e = 0; e < E; ++e) {
      const int32_t c = running[e];
      ws.offsets[e] = acc;
      running[e] = acc;
      acc += c;
    }
    ws.offsets[E] = acc;
    int na = 0;
    for (int e = 0; e < E; ++e)
      if (ws.offsets[e + 1] > ws.offsets[e]) ws.active[na++] = e;
    *ws.nactive = na;
    *ws.ticket = 0;  // ready for the next call
  }
  __syncthreads();
  for (int s = threadIdx.x; s < n; s += kThreads) {
    const int32_t pos = running[ws.ids[s]] + rank[s];
    ws.sorted_slots[pos] = s;
    ws.slot_pos[s] = pos;
    ws.wsorted[pos] = ws.w[s];
  }
}

// Programmatic dependent launch: a kernel's blocks may start while the
// previous kernel of the stream finishes; they wait here for its results.
__device__ __forceinline__ void wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_next_grid() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// --------------------------------------------------------------- gate/up --
// Persistent blocks over items (active expert, 8 rows of F).  Warp w owns
// gate row f and up row f (f = 8*chunk + w): all its 16-byte slices of a
// round (kRV per lane) are requested before any is used, while the expert's
// token rows (<= kRC per pass, gathered from x) are staged in shared memory.
// Rows are then taken one at a time (a short dynamic loop: an expert has
// only a few rows at decode sizes), each dot product reduced across the warp
// at once; partial sums of multi-round rows (H > 2048) live in shared memory.
constexpr int kGUF = kWarps;  // F rows per item (one per warp)
constexpr int kRV = 8;        // 16-byte weight slices per lane per round and row

__global__ void __launch_bounds__(kThreads)
decode_gateup_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w_gate,
                     const __nv_bfloat16* __restrict__ w_up, int T, int H, int F, DecodeWs ws) {
  extern __shared__ uint4 xsm[];  // [kRC][H/8]
  __shared__ float part[kWarps][2][kRC];
  wait_prior_grid();
  allow_next_grid();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hv = H / 8;
  const int nfc = (F + kGUF - 1) / kGUF;
  const int items = *ws.nactive * nfc;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int e = ws.active[item / nfc];
    const int f = (item % nfc) * kGUF + warp;
    const int r0 = ws.offsets[e], cnt = ws.offsets[e + 1] - r0;
    const uint4* wg = reinterpret_cast<const uint4*>(w_gate + ((int64_t)e * F + min(f, F - 1)) * H);
    const uint4* wu = reinterpret_cast<const uint4*>(w_up + ((int64_t)e * F + min(f, F - 1)) * H);
    for (int c0 = 0; c0 < cnt; c0 += kRC) {
      const int rc = min(kRC, cnt - c0);
      uint4 gq[kRV], uq[kRV];
#pragma unroll
      for (int i = 0; i < kRV; ++i) {
        const int v = lane + 32 * i;
        gq[i] = v < hv ? __ldg(wg + v) : make_uint4(0, 0, 0, 0);
        uq[i] = v < hv ? __ldg(wu + v) : make_uint4(0, 0, 0, 0);
      }
      __syncthreads();
      for (int i = threadIdx.x; i < rc * hv; i += kThreads) {
        const int r = i / hv, v = i - r * hv;
        const int t = ws.sorted_slots[r0 + c0 + r] % T;
        xsm[i] = reinterpret_cast<const uint4*>(x + (int64_t)t * H)[v];
      }
      __syncthreads();
      for (int v0 = 0; v0 < hv; v0 += 32 * kRV) {
        if (v0 != 0) {
#pragma unroll
          for (int i = 0; i < kRV; ++i) {
            const int v = v0 + lane + 32 * i;
            gq[i] = v < hv ? __ldg(wg + v) : make_uint4(0, 0, 0, 0);
            uq[i] = v < hv ? __ldg(wu + v) : make_uint4(0, 0, 0, 0);
          }
        }
        for (int r = 0; r < rc; ++r) {
          float g = 0.f, u = 0.f;
#pragma unroll
          for (int i = 0; i < kRV; ++i) {
            const int v = v0 + lane + 32 * i;
            if (v < hv) {
              float gv[8], uv[8], xv[8];
              bf16x8_unpack_here(gq[i], gv);
              bf16x8_unpack_here(uq[i], uv);
              bf16x8_to_f32(xsm[r * hv + v], xv);
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
          if (lane == 0) {
            part[warp][0][r] = (v0 == 0 ? 0.f : part[warp][0][r]) + g;
            part[warp][1][r] = (v0 == 0 ? 0.f : part[warp][1][r]) + u;
          }
        }
      }
      __syncwarp();
      if (lane < rc && f < F) {
        const float g = part[warp][0][lane], u = part[warp][1][lane];
        ws.hs[(int64_t)(r0 + c0 + lane) * F + f] = __float2bfloat16_rn(g * silu_ref(u));
      }
    }
  }
}

// ------------------------------------------------------------------ down --
// Persistent blocks over items (active expert, 32 rows of H): warp w streams
// down rows h0..h0+3 (all slices of a round requested up front) while the
// expert's h rows are staged in shared memory; rows of h one at a time.
// d[row, h] = (down_e[h] . h_row) * gate weight of the row, fp32.
constexpr int kDH = 4;                  // down rows per warp
constexpr int kDItem = kDH * kWarps;    // down rows per item
constexpr int kDV = 4;                  // slices per lane per round and row

__global__ void __launch_bounds__(kThreads)
decode_down_kernel(const __nv_bfloat16* __restrict__ w_down, int H, int F, DecodeWs ws) {
  extern __shared__ uint4 hsm[];  // [kRC][F/8]
  __shared__ float part[kWarps][kDH][kRC];
  wait_prior_grid();
  allow_next_grid();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int fv = F / 8;
  const int nhc = (H + kDItem - 1) / kDItem;
  const int items = *ws.nactive * nhc;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int e = ws.active[item / nhc];
    const int h0 = (item % nhc) * kDItem + warp * kDH;
    const int r0 = ws.offsets[e], cnt = ws.offsets[e + 1] - r0;
    const __nv_bfloat16* wd = w_down + (int64_t)e * H * F;
    for (int c0 = 0; c0 < cnt; c0 += kRC) {
      const int rc = min(kRC, cnt - c0);
      uint4 wq[kDH][kDV];
#pragma unroll
      for (int j = 0; j < kDH; ++j)
#pragma unroll
        for (int i = 0; i < kDV; ++i) {
          const int v = lane + 32 * i;
          wq[j][i] = v < fv ? __ldg(reinterpret_cast<const uint4*>(wd + (int64_t)min(h0 + j, H - 1) * F) + v)
                            : make_uint4(0, 0, 0, 0);
        }
      __syncthreads();
      for (int i = threadIdx.x; i < rc * fv; i += kThreads)
        hsm[i] = reinterpret_cast<const uint4*>(ws.hs + (int64_t)(r0 + c0) * F)[i];
      __syncthreads();
      for (int v0 = 0; v0 < fv; v0 += 32 * kDV) {
        if (v0 != 0) {
#pragma unroll
          for (int j = 0; j < kDH; ++j)
#pragma unroll
            for (int i = 0; i < kDV; ++i) {
              const int v = v0 + lane + 32 * i;
              wq[j][i] = v < fv ? __ldg(reinterpret_cast<const uint4*>(wd + (int64_t)min(h0 + j, H - 1) * F) + v)
                                : make_uint4(0, 0, 0, 0);
            }
        }
        for (int r = 0; r < rc; ++r) {
          float acc[kDH] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int i = 0; i < kDV; ++i) {
            const int v = v0 + lane + 32 * i;
            if (v < fv) {
              float hv8[8];
              bf16x8_to_f32(hsm[r * fv + v], hv8);
#pragma unroll
              for (int j = 0; j < kDH; ++j) {
                float wv[8];
                bf16x8_unpack_here(wq[j][i], wv);
#pragma unroll
                for (int q = 0; q < 8; ++q) acc[j] = fmaf(wv[q], hv8[q], acc[j]);
              }
            }
          }
#pragma unroll
          for (int j = 0; j < kDH; ++j) {
            float v = acc[j];
#pragma unroll
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) part[warp][j][r] = (v0 == 0 ? 0.f : part[warp][j][r]) + v;
          }
        }
      }
      __syncwarp();
      if (lane < kDH * kRC) {
        const int j = lane / kRC, r = lane - j * kRC;
        if (r < rc && h0 + j < H) {
          const int row = r0 + c0 + r;
          ws.d[(int64_t)row * H + h0 + j] = part[warp][j][r] * ws.wsorted[row];
        }
      }
    }
  }
}

// --------------------------------------------------------------- combine --
// y[t, h] = sum_{j<k} d[slot_pos[j*T + t], h] in slot order (deterministic).
template <class TY>
__global__ void __launch_bounds__(kThreads)
decode_combine_kernel(int T, int H, int k, TY* __restrict__ y, DecodeWs ws) {
  wait_prior_grid();
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < (int64_t)T * H;
       i += (int64_t)gridDim.x * kThreads) {
    const int t = (int)(i / H), h = (int)(i - (int64_t)t * H);
    float acc = 0.f;
    for (int j = 0; j < k; ++j) acc += ws.d[(int64_t)ws.slot_pos[j * T + t] * H + h];
    y[i] = from_f32<TY>(acc);
  }
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

}  // namespace

namespace frank {

bool decode_path_ok(int dtype, int64_t T, int64_t H, int64_t F, int64_t E, int64_t k) {
  return dtype == FRANK_BF16 && T >= 1 && T <= 64 && k * T <= kMaxSlots && E <= kMaxE && H % 8 == 0 && F % 8 == 0 &&
         H <= 8192 && F <= 8192;
}

size_t decode_workspace_size(int64_t T, int64_t H, int64_t F, int64_t E, int64_t k) {
  Carve c(nullptr, 0);
  const int64_t n = k * T;
  c.take<float>(E * T);
  c.take<unsigned>(1);
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
  return align_up(c.used, 256);
}

// Writes route_w / route_ids when non-null (copies of the internal buffers).
int launch_decode_block(const void* x, int wr_dtype, const void* wr, const void* w_up_p, const void* w_gate_p,
                        const void* w_down_p, int64_t T, int64_t E, int64_t k, int64_t H, int64_t F, int normalize,
                        int y_dtype, void* y, float* route_w, int32_t* route_ids, void* workspace, size_t ws_bytes,
                        cudaStream_t st, void (*mark)(int, cudaStream_t)) {
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
  ws.ticket = c.take<unsigned>(1);
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
  mark(0, st);
  FRANK_CUDA_TRY(cudaMemsetAsync(ws.ticket, 0, sizeof(unsigned), st));
  const int64_t items = E * ((T + kRouteTok - 1) / kRouteTok);
  const unsigned rblocks = (unsigned)((items + kWarps - 1) / kWarps);
  if (wr_dtype == FRANK_F32)
    decode_route_kernel<float><<<rblocks, kThreads, 0, st>>>((const __nv_bfloat16*)x, (const float*)wr, (int)T,
                                                             (int)H, (int)E, (int)k, normalize, ws);
  else
    decode_route_kernel<__nv_bfloat16><<<rblocks, kThreads, 0, st>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)wr, (int)T, (int)H, (int)E, (int)k, normalize, ws);
  FRANK_LAUNCH_CHECK();
  mark(1, st);
  mark(2, st);
  mark(3, st);
  const int grid_p = num_sms() * 2;
  {
    const size_t smem = (size_t)kRC * H * 2;
    FRANK_CUDA_TRY(cudaFuncSetAttribute(decode_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    FRANK_CUDA_TRY(launch_pdl(decode_gateup_kernel, dim3(grid_p), dim3(kThreads), smem, st,
                              (const __nv_bfloat16*)x, (const __nv_bfloat16*)w_gate_p,
                              (const __nv_bfloat16*)w_up_p, (int)T, (int)H, (int)F, ws));
    FRANK_LAUNCH_CHECK();
  }
  mark(4, st);
  {
    const size_t smem = (size_t)kRC * F * 2;
    FRANK_CUDA_TRY(cudaFuncSetAttribute(decode_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    FRANK_CUDA_TRY(launch_pdl(decode_down_kernel, dim3(grid_p), dim3(kThreads), smem, st,
                              (const __nv_bfloat16*)w_down_p, (int)H, (int)F, ws));
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
  if (route_w) FRANK_CUDA_TRY(cudaMemcpyAsync(route_w, ws.w, n * sizeof(float), cudaMemcpyDeviceToDevice, st));
  if (route_ids)
    FRANK_CUDA_TRY(cudaMemcpyAsync(route_ids, ws.ids, n * sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
  return FRANK_OK;
}

}  // namespace frank
