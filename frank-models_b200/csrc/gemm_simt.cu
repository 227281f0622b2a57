// fp32 grouped GEMM on the FFMA pipe: the FRANK_F32 path.
//
// The reference computes everything in fp32 (tensor<?x?xf32>,
// mul_mat_id.mlir:22-26) and its component tests hold the result to
// rtol 1e-4 / atol 1e-5 (tests/components/test_mul_mat_id.py:30).  TF32
// tensor cores (10-bit mantissa) cannot meet that, so the fp32 path runs on
// CUDA cores.  It serves the reference-shaped tests and the fp32
// configuration (T=32, H=64, F=128); the bf16 path uses tcgen05.
//
//   C[r, n] = sum_k A[r, k] * B_e[n, k]      for rows r of expert e
//   A: expert-sorted activation rows [rows, K]; B: packed weights [E, N, K].
// Epilogues: PLAIN (store), SCALE (multiply row r by wrow[r]),
// SWIGLU (two weight tensors -> gate * silu(up)).
#include "common.cuh"

namespace {

constexpr int BM = 64, BN = 64, BK = 16, THREADS = 256;

enum Epi { PLAIN = 0, SCALE = 1, SWIGLU = 2 };

template <int EPI>
__global__ void __launch_bounds__(THREADS)
grouped_gemm_f32_kernel(const float* __restrict__ A, const float* __restrict__ B, const float* __restrict__ B2,
                        const int32_t* __restrict__ offsets, int E, int64_t N, int64_t K,
                        const float* __restrict__ wrow, float* __restrict__ C) {
  // Find (expert, m-tile) for blockIdx.x: tiles are enumerated expert by
  // expert, ceil(count_e / BM) tiles each.
  __shared__ int s_e, s_m0, s_m1;
  if (threadIdx.x == 0) {
    int acc = 0, e_found = -1, m0 = 0, m1 = 0;
    for (int e = 0; e < E; ++e) {
      int lo = offsets[e], hi = offsets[e + 1];
      int nt = (hi - lo + BM - 1) / BM;
      if ((int)blockIdx.x < acc + nt) {
        e_found = e;
        m0 = lo + ((int)blockIdx.x - acc) * BM;
        m1 = min(hi, m0 + BM);
        break;
      }
      acc += nt;
    }
    s_e = e_found; s_m0 = m0; s_m1 = m1;
  }
  __syncthreads();
  const int e = s_e;
  if (e < 0) return;
  const int m0 = s_m0, m1 = s_m1;
  const int64_t n0 = (int64_t)blockIdx.y * BN;

  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  __shared__ float Bs2[EPI == SWIGLU ? BK : 1][BN + 4];

  const float* Be = B + (int64_t)e * N * K;
  const float* Be2 = EPI == SWIGLU ? B2 + (int64_t)e * N * K : nullptr;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  float acc2[4][4] = {};

  for (int64_t k0 = 0; k0 < K; k0 += BK) {
    for (int i = threadIdx.x; i < BM * BK; i += THREADS) {
      int r = i / BK, c = i % BK;
      int64_t gr = m0 + r, gk = k0 + c;
      As[c][r] = (gr < m1 && gk < K) ? A[gr * K + gk] : 0.f;
    }
    for (int i = threadIdx.x; i < BN * BK; i += THREADS) {
      int r = i / BK, c = i % BK;
      int64_t gn = n0 + r, gk = k0 + c;
      bool ok = gn < N && gk < K;
      Bs[c][r] = ok ? Be[gn * K + gk] : 0.f;
      if constexpr (EPI == SWIGLU) Bs2[c][r] = ok ? Be2[gn * K + gk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], b[4], b2[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        b[j] = Bs[kk][tx * 4 + j];
        if constexpr (EPI == SWIGLU) b2[j] = Bs2[kk][tx * 4 + j];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
          if constexpr (EPI == SWIGLU) acc2[i][j] = fmaf(a[i], b2[j], acc2[i][j]);
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int64_t r = m0 + ty * 4 + i;
    if (r >= m1) continue;
    float s = (EPI == SCALE) ? wrow[r] : 1.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t n = n0 + tx * 4 + j;
      if (n >= N) continue;
      float v = acc[i][j];
      if constexpr (EPI == SWIGLU) v = v * silu_ref(acc2[i][j]);  // B = gate, B2 = up
      if constexpr (EPI == SCALE) v = v * s;
      C[r * N + n] = v;
    }
  }
}

}  // namespace

namespace frank {

// rows: total expert-sorted rows (upper bound for the tile count).
int launch_grouped_gemm_f32(int epi, const float* A, const float* B, const float* B2, const int32_t* offsets,
                            int64_t E, int64_t rows, int64_t N, int64_t K, const float* wrow, float* C,
                            cudaStream_t st) {
  if (rows == 0 || N == 0) return FRANK_OK;
  int64_t mt = (rows + BM - 1) / BM + E;  // >= sum_e ceil(count_e / BM)
  int64_t nt = (N + BN - 1) / BN;
  if (nt > 65535 || mt > 0x7fffffff) {
    set_error("grouped_gemm_f32: grid too large (N=%lld rows=%lld)", (long long)N, (long long)rows);
    return FRANK_EINVAL;
  }
  dim3 grid((unsigned)mt, (unsigned)nt);
  switch (epi) {
    case PLAIN:
      grouped_gemm_f32_kernel<PLAIN><<<grid, THREADS, 0, st>>>(A, B, nullptr, offsets, (int)E, N, K, wrow, C);
      break;
    case SCALE:
      grouped_gemm_f32_kernel<SCALE><<<grid, THREADS, 0, st>>>(A, B, nullptr, offsets, (int)E, N, K, wrow, C);
      break;
    default:
      grouped_gemm_f32_kernel<SWIGLU><<<grid, THREADS, 0, st>>>(A, B, B2, offsets, (int)E, N, K, wrow, C);
  }
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

}  // namespace frank
