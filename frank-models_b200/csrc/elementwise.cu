// Memory-bound kernels around the grouped GEMMs: swiglu, weight prepack,
// row gathers into expert-sorted order, the [O,k,T] output transpose of
// mul_mat_id and the weighted combine.  All are HBM-bound byte movers:
// 128-bit accesses where the layout allows, shared-memory tiles for the
// transposes.
#include "common.cuh"

namespace {

// ------------------------------------------------------------- swiglu ----
// swiglu.mlir:37-47 / oracles/activation.py:11-21: out = g * u / (1 + exp(-u))
template <class T>
__global__ void swiglu_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ o, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float gv = load_as_f32(g, i), uv = load_as_f32(u, i);
    o[i] = from_f32<T>(gv * silu_ref(uv));
  }
}

// ------------------------------------------------------------ prepack ----
// [O, I, E] -> [E, O, I].  For a fixed o the source is an [I, E] row-major
// matrix and the destination an [E, I] one: a 2-D transpose per o through a
// shared-memory tile (mul_mat_id.mlir:38-48 does this on every call; here it
// runs once per weight).
template <class TI, class TO>
__global__ void prepack_kernel(const TI* __restrict__ src, TO* __restrict__ dst, int64_t O, int64_t I, int64_t E) {
  __shared__ float tile[32][33];
  const int64_t o = blockIdx.z;
  const int64_t i0 = (int64_t)blockIdx.x * 32, e0 = (int64_t)blockIdx.y * 32;
  const TI* s = src + o * I * E;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    int64_t i = i0 + r, e = e0 + threadIdx.x;
    tile[r][threadIdx.x] = (i < I && e < E) ? load_as_f32(s, i * E + e) : 0.f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    int64_t e = e0 + r, i = i0 + threadIdx.x;
    if (e < E && i < I) dst[(e * O + o) * I + i] = from_f32<TO>(tile[threadIdx.x][r]);
  }
}

// --------------------------------------------------------- row gather ----
// xs[r, :] = x[sorted_slots[r] % T, :]  (the token of each expert-sorted
// slot; replaces the replicate step moe_ffn_block.mlir:130-144).  One warp
// per row, 16-byte vectors.
__global__ void gather_rows_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ sorted_slots,
                                   int64_t rows, int64_t T, int64_t vec_per_row, uint4* __restrict__ xs) {
  int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (r >= rows) return;
  int64_t t = sorted_slots[r] % T;
  const uint4* src = x + t * vec_per_row;
  uint4* dst = xs + r * vec_per_row;
  for (int64_t v = threadIdx.x & 31; v < vec_per_row; v += 32) dst[v] = src[v];
}

// Scalar fallback for rows whose byte size is not a multiple of 16.
template <class T>
__global__ void gather_rows_scalar_kernel(const T* __restrict__ x, const int32_t* __restrict__ sorted_slots,
                                          int64_t rows, int64_t T_, int64_t H, T* __restrict__ xs) {
  int64_t r = blockIdx.x;
  if (r >= rows) return;
  int64_t t = sorted_slots[r] % T_;
  for (int64_t h = threadIdx.x; h < H; h += blockDim.x) xs[r * H + h] = x[t * H + h];
}

// ------------------------------------------- mul_mat_id input gather ----
// in [I, n_slots] (slot s = j*T + t innermost, mul_mat_id.mlir:24) ->
// xs[r, :] = in[:, sorted_slots[r]].  A transposing gather: a 32x32 tile of
// (rows r, columns i) is read along i per slot and written along i per row.
template <class T>
__global__ void gather_cols_kernel(const T* __restrict__ in, const int32_t* __restrict__ sorted_slots,
                                   int64_t n_slots, int64_t I, T* __restrict__ xs) {
  __shared__ float tile[32][33];
  const int64_t r0 = (int64_t)blockIdx.x * 32, i0 = (int64_t)blockIdx.y * 32;
  // read: thread x walks rows r (slots), y walks i; source in[i, s] -> s scattered
  for (int yy = threadIdx.y; yy < 32; yy += blockDim.y) {
    int64_t i = i0 + yy, r = r0 + threadIdx.x;
    float v = 0.f;
    if (i < I && r < n_slots) v = load_as_f32(in, i * n_slots + sorted_slots[r]);
    tile[threadIdx.x][yy] = v;
  }
  __syncthreads();
  for (int yy = threadIdx.y; yy < 32; yy += blockDim.y) {
    int64_t r = r0 + yy, i = i0 + threadIdx.x;
    if (r < n_slots && i < I) xs[r * I + i] = from_f32<T>(tile[yy][threadIdx.x]);
  }
}

// Tiled form (16-byte vectors; n_slots and I multiples of the vector, 16-byte
// aligned buffers): a block takes 64 slots x 64 columns, reads the 64 input
// rows i along the slot axis (in[i, s0:s0+64], contiguous), transposes them
// through shared memory, and writes each slot's 64 columns into its sorted
// row xs[slot_pos[s], i0:i0+64].  Every global access is a 16-byte vector.
constexpr int kTT = 64;  // tile edge of the tiled transposes

template <class T>
__global__ void __launch_bounds__(256)
gather_cols_tiled_kernel(const T* __restrict__ in, const int32_t* __restrict__ slot_pos, int64_t n_slots,
                         int64_t I, T* __restrict__ xs) {
  constexpr int V = 16 / sizeof(T);  // elements per vector
  constexpr int VR = kTT / V;        // vectors per tile row
  __shared__ float tile[kTT][kTT + 1];  // [slot][column]
  const int64_t s0 = (int64_t)blockIdx.x * kTT, i0 = (int64_t)blockIdx.y * kTT;
  for (int q = threadIdx.x; q < kTT * VR; q += blockDim.x) {
    const int ii = q / VR, v = q - ii * VR;  // input row i0+ii, slots s0+V*v ...
    const int64_t i = i0 + ii, s = s0 + (int64_t)v * V;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (i < I && s < n_slots) u = __ldg(reinterpret_cast<const uint4*>(in + i * n_slots + s));
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < V; ++j) tile[v * V + j][ii] = load_as_f32(e, j);  // exact for bf16 and f32
  }
  __syncthreads();
  for (int q = threadIdx.x; q < kTT * VR; q += blockDim.x) {
    const int ss = q / VR, v = q - ss * VR;  // slot s0+ss, columns i0+V*v ...
    const int64_t s = s0 + ss, i = i0 + (int64_t)v * V;
    if (s >= n_slots || i >= I) continue;
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int j = 0; j < V; ++j) e[j] = from_f32<T>(tile[ss][v * V + j]);
    *reinterpret_cast<uint4*>(xs + (int64_t)slot_pos[s] * I + i) = u;
  }
}

// ---------------------------------------- mul_mat_id output scatter ----
// ys[r, o] (expert-sorted rows) -> out[o, slot] with slot = sorted_slots[r]
// (mul_mat_id.mlir:96-117).  Reads rows through slot_pos so that the write
// side (out[o, s], s innermost) is coalesced.
__global__ void scatter_out_kernel(const float* __restrict__ ys, const int32_t* __restrict__ slot_pos,
                                   int64_t n_slots, int64_t O, float* __restrict__ out) {
  __shared__ float tile[32][33];
  const int64_t s0 = (int64_t)blockIdx.x * 32, o0 = (int64_t)blockIdx.y * 32;
  for (int yy = threadIdx.y; yy < 32; yy += blockDim.y) {
    int64_t s = s0 + yy, o = o0 + threadIdx.x;
    float v = 0.f;
    if (s < n_slots && o < O) v = ys[(int64_t)slot_pos[s] * O + o];
    tile[yy][threadIdx.x] = v;
  }
  __syncthreads();
  for (int yy = threadIdx.y; yy < 32; yy += blockDim.y) {
    int64_t o = o0 + yy, s = s0 + threadIdx.x;
    if (o < O && s < n_slots) out[o * n_slots + s] = tile[threadIdx.x][yy];
  }
}

// Tiled form (n_slots and O multiples of 4, 16-byte aligned buffers): a
// block takes 64 slots x 64 outputs; each slot's row of ys is read as 16
// float4 (256 contiguous bytes), transposed through shared memory, and each
// output row out[o, s0:s0+64] is written as 16 float4.
__global__ void __launch_bounds__(256)
scatter_out_tiled_kernel(const float* __restrict__ ys, const int32_t* __restrict__ slot_pos, int64_t n_slots,
                         int64_t O, float* __restrict__ out) {
  constexpr int VR = kTT / 4;
  __shared__ float tile[kTT][kTT + 1];  // [output][slot]
  const int64_t s0 = (int64_t)blockIdx.x * kTT, o0 = (int64_t)blockIdx.y * kTT;
  for (int q = threadIdx.x; q < kTT * VR; q += blockDim.x) {
    const int ss = q / VR, v = q - ss * VR;  // slot s0+ss, outputs o0+4v ...
    const int64_t s = s0 + ss, o = o0 + 4 * v;
    float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
    if (s < n_slots && o < O) f = __ldg(reinterpret_cast<const float4*>(ys + (int64_t)slot_pos[s] * O + o));
    tile[4 * v + 0][ss] = f.x;
    tile[4 * v + 1][ss] = f.y;
    tile[4 * v + 2][ss] = f.z;
    tile[4 * v + 3][ss] = f.w;
  }
  __syncthreads();
  for (int q = threadIdx.x; q < kTT * VR; q += blockDim.x) {
    const int oo = q / VR, v = q - oo * VR;  // output o0+oo, slots s0+4v ...
    const int64_t o = o0 + oo, s = s0 + 4 * v;
    if (o >= O || s >= n_slots) continue;
    *reinterpret_cast<float4*>(out + o * n_slots + s) =
        make_float4(tile[oo][4 * v], tile[oo][4 * v + 1], tile[oo][4 * v + 2], tile[oo][4 * v + 3]);
  }
}

// -------------------------------------------------------------- combine --
// y[t, :] = sum_{j=0..k-1} d[slot_pos[j*T + t], :]   (moe_ffn_block.mlir:179-206,
// oracles/moe.py:126-132).  The gate weight was already applied by the down
// GEMM epilogue.  Fixed j order, no atomics: deterministic.  4 floats per
// thread; the store is a 16-byte (fp32) or 8-byte (bf16) vector.  With a
// residual (fp32 [T, H], may alias y) the sub-layer's residual add follows
// the sum: y = residual + sum (transformer_layer_moe_prefill.mlir:227-245,
// oracles/transformer_layer.py:123).
template <class TY>
__global__ void combine_kernel(const float* __restrict__ d, const int32_t* __restrict__ slot_pos, int64_t T,
                               int k, int64_t H, TY* y, const float* res) {
  const int64_t t = blockIdx.y;
  const int64_t h = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (h >= H) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < k; ++j) {
    int64_t r = slot_pos[(int64_t)j * T + t];
    float4 v = *reinterpret_cast<const float4*>(d + r * H + h);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  if (res) {
    const float4 rv = *reinterpret_cast<const float4*>(res + t * H + h);
    acc.x = rv.x + acc.x; acc.y = rv.y + acc.y; acc.z = rv.z + acc.z; acc.w = rv.w + acc.w;
  }
  if constexpr (sizeof(TY) == 4) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(y) + t * H + h) = acc;
  } else {
    uint2 p;
    p.x = pack_bf16x2(acc.x, acc.y);
    p.y = pack_bf16x2(acc.z, acc.w);
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(y) + t * H + h) = p;
  }
}

template <class TY>
__global__ void combine_scalar_kernel(const float* __restrict__ d, const int32_t* __restrict__ slot_pos,
                                      int64_t T, int k, int64_t H, TY* y, const float* res) {
  const int64_t t = blockIdx.y;
  for (int64_t h = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; h < H; h += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < k; ++j) acc += d[(int64_t)slot_pos[(int64_t)j * T + t] * H + h];
    if (res) acc = res[t * H + h] + acc;
    y[t * H + h] = from_f32<TY>(acc);
  }
}

// ------------------------------------------------- sorted gate weights ---
__global__ void sorted_weights_kernel(const float* __restrict__ w, const int32_t* __restrict__ sorted_slots,
                                      int64_t n, float* __restrict__ ws) {
  int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r < n) ws[r] = w[sorted_slots[r]];
}

// --------------------------------------------------- row segment copy ----
// dst rows [dst_start[s], +len[s]) = src rows [src_start[s], +len[s]) for
// every segment s; seg_prefix[nseg+1] is the exclusive prefix of len.  One
// warp per destination row (16-byte vectors); the warp finds its segment by
// binary search.  Used by the expert-parallel layer to turn
// source-rank-major received rows into expert-major order and back.
__global__ void copy_row_segments_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                         const int64_t* __restrict__ src_start, const int64_t* __restrict__ dst_start,
                                         const int64_t* __restrict__ seg_prefix, int nseg, int64_t vec_per_row) {
  const int64_t total = seg_prefix[nseg];
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); r < total;
       r += (int64_t)gridDim.x * (blockDim.x / 32)) {
    int lo = 0, hi = nseg;
    while (hi - lo > 1) {
      int mid = (lo + hi) >> 1;
      if (seg_prefix[mid] <= r) lo = mid; else hi = mid;
    }
    const int64_t i = r - seg_prefix[lo];
    const uint4* s = src + (src_start[lo] + i) * vec_per_row;
    uint4* d = dst + (dst_start[lo] + i) * vec_per_row;
    for (int64_t v = lane; v < vec_per_row; v += 32) d[v] = s[v];
  }
}

__global__ void copy_row_segments_u32_kernel(const uint32_t* __restrict__ src, uint32_t* __restrict__ dst,
                                             const int64_t* __restrict__ src_start,
                                             const int64_t* __restrict__ dst_start,
                                             const int64_t* __restrict__ seg_prefix, int nseg, int64_t words) {
  const int64_t total = seg_prefix[nseg] * words;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < total; q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = q / words, wd = q - r * words;
    int lo = 0, hi = nseg;
    while (hi - lo > 1) {
      int mid = (lo + hi) >> 1;
      if (seg_prefix[mid] <= r) lo = mid; else hi = mid;
    }
    const int64_t i = r - seg_prefix[lo];
    dst[(dst_start[lo] + i) * words + wd] = src[(src_start[lo] + i) * words + wd];
  }
}

unsigned grid_1d(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  int64_t cap = (int64_t)frank::num_sms() * 16;
  return (unsigned)(b < cap ? (b < 1 ? 1 : b) : cap);
}

// ------------------------------------------------------------- rms_norm --
// out[t, :] = (x[t, :] / sqrt(mean(x[t, :]^2) + eps)) * w   in fp32, rounded to
// the output type (components/normalization/rms_norm.mlir:18-80,
// oracles/normalization.py:10-43): sum of squares (fused multiply-adds,
// lane partials then a warp tree), divide by H, add eps, sqrt, divide x by
// it, scale by the weight -- the reference's steps, IEEE division and square
// root.  One warp per row; 16-byte loads when H % 4 == 0.
template <class TO>
__global__ void rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ w, int64_t T, int64_t H,
                                float eps, TO* __restrict__ out) {
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const float* xr = x + t * H;
  float ss = 0.f;
  const bool vec = (H % 4 == 0) && ((uintptr_t)xr % 16 == 0);
  if (vec) {
    for (int64_t h = (int64_t)lane * 4; h < H; h += 128) {
      const float4 v = *reinterpret_cast<const float4*>(xr + h);
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
  } else {
    for (int64_t h = lane; h < H; h += 32) ss = fmaf(xr[h], xr[h], ss);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rms = sqrtf(ss / (float)H + eps);
  TO* orow = out + t * H;
  for (int64_t h = lane; h < H; h += 32) orow[h] = from_f32<TO>((xr[h] / rms) * w[h]);
}

}  // namespace

namespace frank {

int launch_swiglu(int dtype, const void* g, const void* u, void* o, int64_t n, cudaStream_t st) {
  if (n == 0) return FRANK_OK;
  if (dtype == FRANK_F32)
    swiglu_kernel<float><<<grid_1d(n, 256), 256, 0, st>>>((const float*)g, (const float*)u, (float*)o, n);
  else
    swiglu_kernel<__nv_bfloat16><<<grid_1d(n, 256), 256, 0, st>>>(
        (const __nv_bfloat16*)g, (const __nv_bfloat16*)u, (__nv_bfloat16*)o, n);
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

int launch_prepack(int in_dtype, const void* src, int64_t O, int64_t I, int64_t E, int out_dtype, void* dst,
                   cudaStream_t st) {
  if (O == 0 || I == 0 || E == 0) return FRANK_OK;
  if (O > 65535) {
    set_error("prepack: O=%lld exceeds 65535", (long long)O);
    return FRANK_EINVAL;
  }
  dim3 grid((unsigned)((I + 31) / 32), (unsigned)((E + 31) / 32), (unsigned)O), block(32, 8);
  if (in_dtype == FRANK_F32 && out_dtype == FRANK_F32)
    prepack_kernel<float, float><<<grid, block, 0, st>>>((const float*)src, (float*)dst, O, I, E);
  else if (in_dtype == FRANK_F32 && out_dtype == FRANK_BF16)
    prepack_kernel<float, __nv_bfloat16><<<grid, block, 0, st>>>((const float*)src, (__nv_bfloat16*)dst, O, I, E);
  else if (in_dtype == FRANK_BF16 && out_dtype == FRANK_BF16)
    prepack_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, block, 0, st>>>((const __nv_bfloat16*)src,
                                                                        (__nv_bfloat16*)dst, O, I, E);
  else {
    set_error("prepack: unsupported dtype pair %d -> %d", in_dtype, out_dtype);
    return FRANK_EINVAL;
  }
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

int launch_gather_rows(int dtype, const void* x, const int32_t* sorted_slots, int64_t rows, int64_t T, int64_t H,
                       void* xs, cudaStream_t st) {
  if (rows == 0) return FRANK_OK;
  size_t esz = dtype == FRANK_F32 ? 4 : 2;
  size_t row_bytes = H * esz;
  bool vec_ok = (row_bytes % 16 == 0) && ((uintptr_t)x % 16 == 0) && ((uintptr_t)xs % 16 == 0);
  if (vec_ok) {
    gather_rows_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>((const uint4*)x, sorted_slots, rows, T,
                                                                   (int64_t)(row_bytes / 16), (uint4*)xs);
  } else if (dtype == FRANK_F32) {
    gather_rows_scalar_kernel<float><<<(unsigned)rows, 128, 0, st>>>((const float*)x, sorted_slots, rows, T, H,
                                                                     (float*)xs);
  } else {
    gather_rows_scalar_kernel<__nv_bfloat16><<<(unsigned)rows, 128, 0, st>>>(
        (const __nv_bfloat16*)x, sorted_slots, rows, T, H, (__nv_bfloat16*)xs);
  }
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

// slot_pos (may be null): the tiled form's inverse of sorted_slots.
int launch_gather_cols(int dtype, const void* in, const int32_t* sorted_slots, int64_t n_slots, int64_t I, void* xs,
                       cudaStream_t st, const int32_t* slot_pos) {
  if (n_slots == 0 || I == 0) return FRANK_OK;
  const int64_t vec = dtype == FRANK_F32 ? 4 : 8;
  if (slot_pos && n_slots % vec == 0 && I % vec == 0 && (uintptr_t)in % 16 == 0 && (uintptr_t)xs % 16 == 0 &&
      (I + kTT - 1) / kTT <= 65535) {
    dim3 grid((unsigned)((n_slots + kTT - 1) / kTT), (unsigned)((I + kTT - 1) / kTT));
    if (dtype == FRANK_F32)
      gather_cols_tiled_kernel<float><<<grid, 256, 0, st>>>((const float*)in, slot_pos, n_slots, I, (float*)xs);
    else
      gather_cols_tiled_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)in, slot_pos, n_slots,
                                                                     I, (__nv_bfloat16*)xs);
    FRANK_LAUNCH_CHECK();
    return FRANK_OK;
  }
  if ((I + 31) / 32 > 65535) {
    set_error("gather_cols: I=%lld too large", (long long)I);
    return FRANK_EINVAL;
  }
  dim3 grid((unsigned)((n_slots + 31) / 32), (unsigned)((I + 31) / 32)), block(32, 8);
  if (dtype == FRANK_F32)
    gather_cols_kernel<float><<<grid, block, 0, st>>>((const float*)in, sorted_slots, n_slots, I, (float*)xs);
  else
    gather_cols_kernel<__nv_bfloat16><<<grid, block, 0, st>>>((const __nv_bfloat16*)in, sorted_slots, n_slots, I,
                                                              (__nv_bfloat16*)xs);
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

int launch_scatter_out(const float* ys, const int32_t* slot_pos, int64_t n_slots, int64_t O, float* out,
                       cudaStream_t st) {
  if (n_slots == 0 || O == 0) return FRANK_OK;
  if (n_slots % 4 == 0 && O % 4 == 0 && (uintptr_t)ys % 16 == 0 && (uintptr_t)out % 16 == 0 &&
      (O + kTT - 1) / kTT <= 65535) {
    dim3 grid((unsigned)((n_slots + kTT - 1) / kTT), (unsigned)((O + kTT - 1) / kTT));
    scatter_out_tiled_kernel<<<grid, 256, 0, st>>>(ys, slot_pos, n_slots, O, out);
    FRANK_LAUNCH_CHECK();
    return FRANK_OK;
  }
  if ((O + 31) / 32 > 65535) {
    set_error("scatter_out: O=%lld too large", (long long)O);
    return FRANK_EINVAL;
  }
  dim3 grid((unsigned)((n_slots + 31) / 32), (unsigned)((O + 31) / 32)), block(32, 8);
  scatter_out_kernel<<<grid, block, 0, st>>>(ys, slot_pos, n_slots, O, out);
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

int launch_combine(int dtype, const float* d, const int32_t* slot_pos, int64_t T, int64_t k, int64_t H, void* y,
                   cudaStream_t st, const float* residual) {
  if (T == 0 || H == 0) return FRANK_OK;
  bool vec_ok = (H % 4 == 0) && ((uintptr_t)d % 16 == 0) &&
                ((uintptr_t)y % (dtype == FRANK_F32 ? 16 : 8) == 0) && ((uintptr_t)residual % 16 == 0);
  for (int64_t t0 = 0; t0 < T; t0 += 65535) {
    int64_t tn = (T - t0) < 65535 ? (T - t0) : 65535;
    // Offsetting y and slot_pos by t0 keeps each launch within grid.y limits;
    // slot_pos is indexed j*T + t, so pass the base and let t run from t0.
    if (vec_ok) {
      dim3 grid((unsigned)((H / 4 + 127) / 128), (unsigned)tn);
      if (dtype == FRANK_F32)
        combine_kernel<float><<<grid, 128, 0, st>>>(d, slot_pos + t0, T, (int)k, H, (float*)y + t0 * H,
                                                    residual ? residual + t0 * H : nullptr);
      else
        combine_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(d, slot_pos + t0, T, (int)k, H,
                                                            (__nv_bfloat16*)y + t0 * H,
                                                            residual ? residual + t0 * H : nullptr);
    } else {
      dim3 grid((unsigned)((H + 127) / 128 < 64 ? (H + 127) / 128 : 64), (unsigned)tn);
      if (dtype == FRANK_F32)
        combine_scalar_kernel<float><<<grid, 128, 0, st>>>(d, slot_pos + t0, T, (int)k, H, (float*)y + t0 * H,
                                                           residual ? residual + t0 * H : nullptr);
      else
        combine_scalar_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(d, slot_pos + t0, T, (int)k, H,
                                                                   (__nv_bfloat16*)y + t0 * H,
                                                                   residual ? residual + t0 * H : nullptr);
    }
    FRANK_LAUNCH_CHECK();
  }
  return FRANK_OK;
}

int launch_copy_row_segments(const void* src, void* dst, const int64_t* src_start, const int64_t* dst_start,
                             const int64_t* seg_prefix, int64_t nseg, int64_t total_rows, int64_t row_bytes,
                             cudaStream_t st) {
  if (total_rows == 0 || nseg == 0) return FRANK_OK;
  if (row_bytes % 4 != 0) {
    set_error("copy_row_segments: row_bytes=%lld is not a multiple of 4", (long long)row_bytes);
    return FRANK_EINVAL;
  }
  const int64_t cap = (int64_t)num_sms() * 16;
  if (row_bytes % 16 == 0 && (uintptr_t)src % 16 == 0 && (uintptr_t)dst % 16 == 0) {
    int64_t blocks = (total_rows + 7) / 8;
    copy_row_segments_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, st>>>(
        (const uint4*)src, (uint4*)dst, src_start, dst_start, seg_prefix, (int)nseg, row_bytes / 16);
  } else {
    int64_t words = row_bytes / 4;
    int64_t blocks = (total_rows * words + 255) / 256;
    copy_row_segments_u32_kernel<<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, st>>>(
        (const uint32_t*)src, (uint32_t*)dst, src_start, dst_start, seg_prefix, (int)nseg, words);
  }
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

int launch_sorted_weights(const float* w, const int32_t* sorted_slots, int64_t n, float* ws, cudaStream_t st) {
  if (n == 0) return FRANK_OK;
  sorted_weights_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, sorted_slots, n, ws);
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

int launch_rms_norm(const float* x, const float* w, int64_t T, int64_t H, float eps, int out_dtype, void* out,
                    cudaStream_t st) {
  if (T == 0) return FRANK_OK;
  const unsigned blocks = (unsigned)((T + 3) / 4);
  if (out_dtype == FRANK_F32)
    rms_norm_kernel<float><<<blocks, 128, 0, st>>>(x, w, T, H, eps, (float*)out);
  else
    rms_norm_kernel<__nv_bfloat16><<<blocks, 128, 0, st>>>(x, w, T, H, eps, (__nv_bfloat16*)out);
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

}  // namespace frank
