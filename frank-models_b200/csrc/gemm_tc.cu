// Grouped expert GEMM on the 5th-generation tensor cores (tcgen05 + TMEM),
// fed by TMA: the bf16 path of mul_mat_id and moe_ffn_block.
//
//   C[r, n] = sum_k A[r, k] * B_e[n, k]   for the rows r of expert e
//   A  : expert-sorted activation rows [rows, K] bf16 (K-major)
//   B_e: packed expert weights [E, N, K] bf16 (K-major)
//
// Replaces the gather of whole expert matrices + per-slot mat-vec of
// components/moe/mul_mat_id.mlir:58-94 (oracles/moe.py:33-44) with one
// GEMM per expert over the rows routed to it.
//
// Structure (one persistent CTA per SM, 192 threads, 1 CTA/SM):
//   warp 0      TMA producer: A tile 128x64 + B tile 256x64 per stage
//               (SWIZZLE_128B), 4-stage mbarrier ring.
//   warp 1      TMEM allocator + MMA issuer: tcgen05.mma.cta_group::1
//               kind::f16, M=128 N=256 K=16, fp32 accumulator in TMEM,
//               two accumulator buffers (2 x 256 columns).
//   warps 2..5  epilogue: tcgen05.ld 32x32b, fused activation, stores.
// Tiles are (expert, m-tile, n-tile) with m fastest inside an expert so the
// CTAs running at the same time share weight tiles through L2; the per-
// expert tile prefix is computed on the device from the permutation's
// offsets, so the host never synchronises.
//
// Epilogue modes
//   SWIGLU: B tile = 128 gate rows + 128 up rows of the same n range; the
//           epilogue writes h = gate * silu(up) as bf16 [rows, N]
//           (swiglu.mlir:37-47, silu on `up`).
//   SCALE : 256 output columns scaled by the row's gate weight, fp32 out
//           (moe_ffn_block.mlir:162-177).
//   PLAIN : 256 output columns, fp32 out (mul_mat_id).
// Every mbarrier wait is bounded (about 2 s); on expiry the CTA records
// FRANK_ETIMEOUT in the device error word and unwinds, freeing its TMEM.
#include <cuda.h>
#include <cstdlib>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "mbarrier.cuh"

namespace {
using namespace frank_mbar;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, THREADS = 192;
constexpr uint32_t A_BYTES = BM * BK * 2;        // 16 KiB
constexpr uint32_t B_HALF_BYTES = 128 * BK * 2;  // 16 KiB
constexpr uint32_t B_BYTES = BN * BK * 2;        // 32 KiB
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t EPI_STAGE_BYTES = 4 * 32 * 128;  // epilogue staging, 4 KiB per epilogue warp
constexpr int kMaxExperts = 1024;
constexpr int kMaxPeers = 8;

enum Mode { SWIGLU = 0, SCALE = 1, PLAIN = 2 };

struct Params {
  const int32_t* offsets;  // [E+1] expert row offsets (permutation output); null: one group of `rows`
  int E;
  int rows;                // total rows (used when offsets is null, E == 1)
  int n_tiles;             // output column tiles per expert
  int N_out;               // output columns
  int K;
  void* out;               // SWIGLU: bf16 [rows, ldo]; SCALE/PLAIN: fp32 [rows, ldo]
  int64_t ldo;
  const float* wrow;       // SCALE: per sorted row weight
  int32_t* err;            // device error word
  // SCALE with a row map: row r goes to peer_out[row_rank[r]] + row_pos[r] * ldo
  // (another GPU's buffer reached over NVLink) instead of out + r * ldo.
  const int32_t* row_rank;
  const int32_t* row_pos;
  float* peer_out[kMaxPeers];
  int band_rows;           // rows per L2-resident band of activation rows
  int n_peers;             // entries of peer_out in use
  int64_t peer_rows;       // rows of every peer's return buffer
  int swap_small;          // experts with <= BM rows run as swapped (weight-row-major) tiles
};

// Destination of row `row` under a row map: another rank's return buffer.
// A map entry outside [0, n_peers) x [0, peer_rows) is refused (nullptr, the
// row is not stored) and recorded in the device error word.
__device__ __forceinline__ float* mapped_row(const Params& p, int row) {
  const int32_t q = p.row_rank[row], pos = p.row_pos[row];
  if (q < 0 || q >= p.n_peers || pos < 0 || (int64_t)pos >= p.peer_rows || p.peer_out[q] == nullptr) {
    atomicExch(p.err, FRANK_EINVAL);
    return nullptr;
  }
  return p.peer_out[q] + (int64_t)pos * p.ldo;
}

// ------------------------------------------------------------ PTX glue --
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart.
// Fields: start>>4 [0,14), LBO>>4 [16,30) (=1, unused for swizzled K-major),
// SBO>>4 [32,46) (=1024>>4), version 1 [46,48), layout SWIZZLE_128B=2 [61,64).
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: D fp32 [4,6)=1, A bf16 [7,10)=1,
// B bf16 [10,13)=1, both K-major, N>>3 at [17,23), M>>4 at [24,29).
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

// Same with a run-time instruction descriptor (swapped tiles: M = 128
// weight rows, N = the expert's token rows rounded up to 16).
__device__ __forceinline__ void mma_bf16_i(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------- kernel --
// Activation rows of one band kept resident in L2 (a band's A rows are
// read once while the CTAs sweep the weight tiles): about 64 MB.
constexpr int64_t kBandBytes = 64ll << 20;

// swapN != 0: a swapped tile.  The expert has at most BM rows, so the MMAs
// run with the 128 weight rows of each B half as M and the expert's token
// rows (rounded up to 16) as N: D0 = (B rows 0-127) x tokens in TMEM columns
// [0, swapN), D1 = (B rows 128-255) x tokens in [swapN, 2 swapN).  The
// shared-memory tiles are the normal ones; the MMA work falls to swapN/128
// of a normal tile's.
struct Tile {
  int e, m0, m_end, n, swapN;
};

// Row offset of group e (offsets[e], or 0 / rows for the single-group form).
__device__ __forceinline__ int off_at(const Params& p, int e) {
  return p.offsets != nullptr ? p.offsets[e] : (e == 0 ? 0 : p.rows);
}

__device__ __forceinline__ Tile decode_tile(int t, const int* prefix, const Params& p, int bm = BM,
                                            bool allow_swap = false) {
  int lo = 0, hi = p.E;  // find e: prefix[e] <= t < prefix[e+1]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (prefix[mid] <= t) lo = mid; else hi = mid;
  }
  const int e = lo;
  const int r0 = off_at(p, e), r1 = off_at(p, e + 1);
  const int mt = (r1 - r0 + bm - 1) / bm;
  const int nt = (prefix[e + 1] - prefix[e]) / mt;
  const int local = t - prefix[e];
  // Bands of p.band_rows rows (L2-resident: band_rows x K bf16 <= 64 MB);
  // inside a band m runs fastest, so the CTAs running at the same time share
  // both the band's activation rows and a few weight tiles, and each weight
  // tile is read from HBM once per band.
  const int G = max(1, p.band_rows / bm);
  const int band = local / (G * nt);
  const int gm = min(G, mt - band * G);
  const int in = local - band * G * nt;
  Tile tl;
  tl.e = e;
  tl.m0 = r0 + (band * G + in % gm) * bm;
  tl.m_end = r1;
  tl.n = in / gm;
  tl.swapN = (allow_swap && mt == 1) ? ((r1 - r0 + 15) & ~15) : 0;
  return tl;
}

// Epilogue of one accumulator tile for the 32 rows of one warp: thread
// `lane` owns row `row`; taddr addresses this warp's TMEM lane quadrant.
// Epilogue of one accumulator tile for this warp's 32 rows (row: this lane's
// row).  Values pass through a per-warp shared-memory stage of 32 rows x
// 128 bytes (16-byte chunk c of row r kept at chunk c ^ (r & 7), so the
// row-per-lane writes and the row-wise reads are both free of bank
// conflicts): each global store instruction then covers 4 rows x 128
// contiguous bytes instead of 32 rows x 16 bytes.
template <int MODE>
__device__ __forceinline__ void epilogue_rows(const Params& p, int row, bool valid, int n, uint32_t taddr,
                                              uint4* stage) {
  const int lane = threadIdx.x & 31;
  const uint32_t sw = (uint32_t)(lane & 7);
  // byte address of this lane's row at the tile's first column (0: no row)
  unsigned long long my = 0ull;
  if (MODE == SWIGLU) {
    if (valid)
      my = (unsigned long long)(reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)row * p.ldo + n * 128);
  } else if (valid) {
    float* out = MODE == SCALE && p.row_rank != nullptr ? mapped_row(p, row)
                                                        : reinterpret_cast<float*>(p.out) + (int64_t)row * p.ldo;
    if (out != nullptr) my = (unsigned long long)(out + n * BN);
  }
  // stage -> global: 8 rounds of 4 rows x 8 chunks; chunk_cols columns per
  // 16-byte chunk; col0: the stage's first column within the tile
  auto flush = [&](int col0, int chunk_cols, int elem_bytes) {
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = i * 4 + (lane >> 3), c = lane & 7;
      const unsigned long long base = __shfl_sync(0xffffffffu, my, r);
      const uint4 v = stage[r * 8 + (c ^ (r & 7))];
      const int col = (MODE == SWIGLU ? n * 128 : n * BN) + col0 + c * chunk_cols;
      if (base != 0ull && col < p.N_out)
        *reinterpret_cast<uint4*>(base + (unsigned long long)(col0 + c * chunk_cols) * elem_bytes) = v;
    }
    __syncwarp();
  };
  if (MODE == SWIGLU) {
#pragma unroll 1
    for (int c = 0; c < 128; c += 64) {
#pragma unroll 1
      for (int sub = 0; sub < 64; sub += 16) {
        float g[16], u[16];
        tmem_ld16(taddr + c + sub, g);
        tmem_ld16(taddr + 128 + c + sub, u);
        tmem_wait_ld();
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          pk[i] = pack_bf16x2(g[2 * i] * silu_ref(u[2 * i]), g[2 * i + 1] * silu_ref(u[2 * i + 1]));
        const uint32_t j = (uint32_t)(sub >> 3);
        stage[lane * 8 + (j ^ sw)] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        stage[lane * 8 + ((j + 1) ^ sw)] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
      flush(c, 8, 2);
    }
  } else {
    const float s = (MODE == SCALE && valid) ? p.wrow[row] : 1.f;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float v[32];
      tmem_ld16(taddr + c, *reinterpret_cast<float(*)[16]>(v));
      tmem_ld16(taddr + c + 16, *reinterpret_cast<float(*)[16]>(v + 16));
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 8; ++j)
        stage[lane * 8 + ((uint32_t)j ^ sw)] =
            make_uint4(__float_as_uint(v[4 * j] * s), __float_as_uint(v[4 * j + 1] * s),
                       __float_as_uint(v[4 * j + 2] * s), __float_as_uint(v[4 * j + 3] * s));
      flush(c, 4, 4);
    }
  }
}

// Epilogue of a swapped tile: this lane owns weight row wr (0..127) of both
// accumulators, i.e. output column n*128 + wr (SWIGLU: gate in D0, up in D1)
// or n*BN + wr and n*BN + 128 + wr (SCALE / PLAIN), for each of the
// expert's token rows.  Per token the 32 lanes of a warp store 32
// consecutive columns (64 or 128 contiguous bytes).
template <int MODE>
__device__ __forceinline__ void epilogue_swapped(const Params& p, const Tile& tl, int wr, uint32_t taddr) {
  const int rows = tl.m_end - tl.m0;
  const int N = tl.swapN;
#pragma unroll 1
  for (int t0 = 0; t0 < N; t0 += 16) {
    float v0[16], v1[16];
    tmem_ld16(taddr + t0, v0);
    tmem_ld16(taddr + N + t0, v1);
    tmem_wait_ld();
    const int nt = min(16, rows - t0);
    if (MODE == SWIGLU) {
      const int col = tl.n * 128 + wr;
      if (col < p.N_out) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out) + col;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (i < nt) out[(int64_t)(tl.m0 + t0 + i) * p.ldo] = __float2bfloat16_rn(v0[i] * silu_ref(v1[i]));
      }
    } else {
      const int c0 = tl.n * BN + wr, c1 = c0 + 128;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (i < nt) {
          const int row = tl.m0 + t0 + i;
          float* out = MODE == SCALE && p.row_rank != nullptr
                           ? mapped_row(p, row)
                           : reinterpret_cast<float*>(p.out) + (int64_t)row * p.ldo;
          const float sc = MODE == SCALE ? p.wrow[row] : 1.f;
          if (out != nullptr && c0 < p.N_out) out[c0] = v0[i] * sc;
          if (out != nullptr && c1 < p.N_out) out[c1] = v1[i] * sc;
        }
      }
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1)
tc_grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ CUtensorMap tmA16,
                       const __grid_constant__ CUtensorMap tmA32, const __grid_constant__ CUtensorMap tmA64,
                       const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint4* epi_stage = reinterpret_cast<uint4*>(smem + STAGES * STAGE_BYTES);  // [4 warps][32 rows][8 chunks]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES + EPI_STAGE_BYTES);
  // bars[0..S) full, [S..2S) empty, [2S, 2S+2) tmem_full, [2S+2, 2S+4) tmem_empty
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* prefix = reinterpret_cast<int*>(tmem_slot + 4);  // [E+1]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0) {
    // tile prefix over experts: prefix[e] = sum_{e'<e} ceil(cnt_e'/BM) * n_tiles
    int carry = 0;
    for (int base = 0; base < p.E; base += 32) {
      int e = base + lane;
      int v = 0;
      if (e < p.E) v = ((off_at(p, e + 1) - off_at(p, e) + BM - 1) / BM) * p.n_tiles;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      if (e < p.E) prefix[e] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) prefix[p.E] = carry;
  } else if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = prefix[p.E];
  const int nk = (p.K + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer --
      uint32_t it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        Tile tl = decode_tile(t, prefix, p, BM, p.swap_small != 0);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
          uint8_t* st = smem + s * STAGE_BYTES;
          // swapped tiles read only the expert's rows: a 16/32/64-row A box
          const int arows = tl.swapN == 0 ? BM : tl.swapN <= 16 ? 16 : tl.swapN <= 32 ? 32 : tl.swapN <= 64 ? 64 : BM;
          const CUtensorMap* mapA = arows == 16 ? &tmA16 : arows == 32 ? &tmA32 : arows == 64 ? &tmA64 : &tmA;
          mbar_expect_tx(full_bar(s), (uint32_t)arows * BK * 2 + B_BYTES);
          tma_load_2d(smem_u32(st), mapA, kb * BK, tl.m0, full_bar(s));
          if (MODE == SWIGLU) {
            tma_load_3d(smem_u32(st + A_BYTES), &tmB, kb * BK, tl.n * 128, tl.e, full_bar(s));
            tma_load_3d(smem_u32(st + A_BYTES + B_HALF_BYTES), &tmB2, kb * BK, tl.n * 128, tl.e, full_bar(s));
          } else {
            tma_load_3d(smem_u32(st + A_BYTES), &tmB, kb * BK, tl.n * BN, tl.e, full_bar(s));
            tma_load_3d(smem_u32(st + A_BYTES + B_HALF_BYTES), &tmB, kb * BK, tl.n * BN + 128, tl.e, full_bar(s));
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------- MMA issuer --
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++tc) {
        const uint32_t a = tc & 1u, aph = (tc >> 1) & 1u;
        if (!mbar_wait(tempty_bar(a), aph ^ 1u, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + a * BN;
        const int swapN = p.swap_small ? decode_tile(t, prefix, p, BM, true).swapN : 0;
        const uint32_t idesc_sw =
            (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(swapN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(full_bar(s), ph, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
          const uint64_t adesc = make_sw128_desc(sa);
          const uint64_t bdesc = make_sw128_desc(sa + A_BYTES);
          if (swapN == 0) {
#pragma unroll
            for (int j = 0; j < BK / 16; ++j) {
              // advance 16 bf16 = 32 B along K inside the 128-B swizzle row
              mma_bf16(d, adesc + (uint64_t)(2 * j), bdesc + (uint64_t)(2 * j), (kb | j) != 0);
            }
          } else {
            const uint64_t b1desc = make_sw128_desc(sa + A_BYTES + B_HALF_BYTES);
#pragma unroll
            for (int j = 0; j < BK / 16; ++j) {
              mma_bf16_i(d, bdesc + (uint64_t)(2 * j), adesc + (uint64_t)(2 * j), idesc_sw, (kb | j) != 0);
              mma_bf16_i(d + (uint32_t)swapN, b1desc + (uint64_t)(2 * j), adesc + (uint64_t)(2 * j), idesc_sw,
                         (kb | j) != 0);
            }
          }
          mma_commit(empty_bar(s));
        }
        if (ok) mma_commit(tfull_bar(a));
      }
    }
  } else {
    // ------------------------------------------------------ epilogue --
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    uint32_t tc = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++tc) {
      Tile tl = decode_tile(t, prefix, p, BM, p.swap_small != 0);
      const uint32_t a = tc & 1u, aph = (tc >> 1) & 1u;
      if (!mbar_wait(tfull_bar(a), aph, abort_flag, p.err)) break;
      tc_fence_after();
      const int row = tl.m0 + q * 32 + lane;
      if (tl.swapN)
        epilogue_swapped<MODE>(p, tl, q * 32 + lane, tmem_base + a * BN + ((uint32_t)(q * 32) << 16));
      else
        epilogue_rows<MODE>(p, row, row < tl.m_end, tl.n, tmem_base + a * BN + ((uint32_t)(q * 32) << 16),
                            epi_stage + q * 256);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(a));
    }
    // rows stored into other GPUs' memory must be visible to them once this
    // kernel has completed
    if (MODE == SCALE && p.row_rank != nullptr) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------- CTA-pair (2-SM) form --
// Same grouped GEMM with tcgen05.mma.cta_group::2: a cluster of two CTAs on
// two SMs computes a 256-row x 256-column tile.  Each CTA loads its own
// 128 rows of A and its half of B (128 rows: for SWIGLU the gate rows in
// CTA 0 and the up rows in CTA 1), so per SM the shared-memory operand traffic
// per MMA drops from 48 KB to 32 KB per 64-wide K step.  CTA 0 (the leader)
// issues the MMAs; each CTA's TMEM holds the accumulator rows of its 128 A
// rows, and both run the same epilogue on their rows.  TMA loads of both CTAs
// signal the leader's full barrier (.cta_group::2 form, no multicast);
// tcgen05.commit multicasts stage-free and accumulator-ready arrivals to both
// CTAs; the peer's epilogue warps arrive on the leader's accumulator-free
// barrier through its cluster address.
constexpr int BM2 = 256;
constexpr int STAGES2 = 6;
constexpr uint32_t STAGE2_BYTES = A_BYTES + B_HALF_BYTES;  // 32 KiB per CTA
constexpr uint32_t kIdesc2 =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM2 >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4}], [%5];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(kIdesc2), "r"(accumulate)
      : "memory");
}

// arrive on the barrier at this shared offset in both CTAs of the pair
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"((uint16_t)3)
      : "memory");
}

template <int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
tc2_grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmB2, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint4* epi_stage = reinterpret_cast<uint4*>(smem + STAGES2 * STAGE2_BYTES);  // [4 warps][32 rows][8 chunks]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES2 * STAGE2_BYTES + EPI_STAGE_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES2 + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* prefix = reinterpret_cast<int*>(tmem_slot + 4);  // [E+1]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES2 + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES2 + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES2 + 2 + a); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 8);  // 4 epilogue warps in each CTA of the pair
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < p.E; base += 32) {
      int e = base + lane;
      int v = 0;
      if (e < p.E) v = ((off_at(p, e + 1) - off_at(p, e) + BM2 - 1) / BM2) * p.n_tiles;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      if (e < p.E) prefix[e] = carry + incl - v;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) prefix[p.E] = carry;
  } else if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers are initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = prefix[p.E];
  const int nk = (p.K + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------- TMA producer (both CTAs) --
      uint32_t it = 0;
      bool ok = true;
      for (int t = cid; t < total && ok; t += ncl) {
        Tile tl = decode_tile(t, prefix, p, BM2);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES2;
          const uint32_t ph = (it / STAGES2) & 1u;
          if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
          uint8_t* st = smem + s * STAGE2_BYTES;
          if (leader) mbar_expect_tx(full_bar(s), 2 * STAGE2_BYTES);
          const uint32_t fb = mapa_shared(full_bar(s), 0);
          tma_load_2d_pair(smem_u32(st), &tmA, kb * BK, tl.m0 + (int)rank * 128, fb);
          if (MODE == SWIGLU)
            tma_load_3d_pair(smem_u32(st + A_BYTES), rank == 0 ? &tmB : &tmB2, kb * BK, tl.n * 128, tl.e, fb);
          else
            tma_load_3d_pair(smem_u32(st + A_BYTES), &tmB, kb * BK, tl.n * BN + (int)rank * 128, tl.e, fb);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // -------------------------------------------- MMA issuer (leader) --
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int t = cid; t < total && ok; t += ncl, ++tc) {
        const uint32_t a = tc & 1u, aph = (tc >> 1) & 1u;
        if (!mbar_wait(tempty_bar(a), aph ^ 1u, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + a * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES2;
          const uint32_t ph = (it / STAGES2) & 1u;
          if (!mbar_wait(full_bar(s), ph, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * STAGE2_BYTES);
          const uint64_t adesc = make_sw128_desc(sa);
          const uint64_t bdesc = make_sw128_desc(sa + A_BYTES);
#pragma unroll
          for (int j = 0; j < BK / 16; ++j)
            mma_bf16_pair(d, adesc + (uint64_t)(2 * j), bdesc + (uint64_t)(2 * j), (kb | j) != 0);
          mma_commit_pair(empty_bar(s));
        }
        if (ok) mma_commit_pair(tfull_bar(a));
      }
    }
  } else {
    // ------------------------------------------- epilogue (both CTAs) --
    const int q = warp & 3;
    uint32_t tc = 0;
    for (int t = cid; t < total; t += ncl, ++tc) {
      Tile tl = decode_tile(t, prefix, p, BM2);
      const uint32_t a = tc & 1u, aph = (tc >> 1) & 1u;
      if (!mbar_wait(tfull_bar(a), aph, abort_flag, p.err)) break;
      tc_fence_after();
      const int row = tl.m0 + (int)rank * 128 + q * 32 + lane;
      epilogue_rows<MODE>(p, row, row < tl.m_end, tl.n, tmem_base + a * BN + ((uint32_t)(q * 32) << 16),
                          epi_stage + q * 256);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty_bar(a), 0));
    }
    if (MODE == SCALE && p.row_rank != nullptr) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's MMAs read the peer's shared memory until here
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------ host side --
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2-D bf16 map [rows, K], box {64, 128}, 128-B swizzle.
int make_map_2d(CUtensorMap* m, const void* base, int64_t rows, int64_t K, uint32_t box_rows = 128) {
  auto enc = get_encode();
  if (!enc) {
    frank::set_error("cuTensorMapEncodeTiled unavailable");
    return FRANK_ECUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {BK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    frank::set_error("cuTensorMapEncodeTiled(2d rows=%lld K=%lld) failed: %d", (long long)rows, (long long)K, (int)r);
    return FRANK_ECUDA;
  }
  return FRANK_OK;
}

// 3-D bf16 map [E, N, K], box {64, 128, 1}, 128-B swizzle.
int make_map_3d(CUtensorMap* m, const void* base, int64_t E, int64_t N, int64_t K) {
  auto enc = get_encode();
  if (!enc) {
    frank::set_error("cuTensorMapEncodeTiled unavailable");
    return FRANK_ECUDA;
  }
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)N, (cuuint64_t)E};
  cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)N * K * 2};
  cuuint32_t box[3] = {BK, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    frank::set_error("cuTensorMapEncodeTiled(3d E=%lld N=%lld K=%lld) failed: %d", (long long)E, (long long)N,
                     (long long)K, (int)r);
    return FRANK_ECUDA;
  }
  return FRANK_OK;
}

size_t smem_bytes(int E) {
  return 1024 + STAGES * STAGE_BYTES + EPI_STAGE_BYTES + 8 * (2 * STAGES + 4) + 16 + 4 * (E + 1) + 64;
}
size_t smem2_bytes(int E) {
  return 1024 + STAGES2 * STAGE2_BYTES + EPI_STAGE_BYTES + 8 * (2 * STAGES2 + 4) + 16 + 4 * (E + 1) + 64;
}

// The CTA-pair form is opt-in (FRANK_TC_PAIR=1): on the B200s measured it
// was ~7% slower than the single-CTA kernel on the Mixtral block, whose
// GEMMs run at the 1 kW power cap (about 90% of the sustained cuBLAS rate),
// not at a shared-memory limit.
// The CTA-pair form moves 32 KB instead of 48 KB into each SM's shared
// memory per 64-wide K step, so the same ring covers 1.6 us of TMA latency
// instead of about 1 us; measured on the Mixtral block (C3) it runs the
// gate/up GEMM 4% and the down GEMM 7% faster.  Its 256-row tiles waste
// work on small experts (it has no swapped form), so it is chosen when the
// experts average at least 1024 rows.  FRANK_TC_PAIR=0/1 forces either form.
bool use_cta_pair(int64_t rows, int64_t E) {
  static int force = -2;
  if (force == -2) {
    const char* v = getenv("FRANK_TC_PAIR");
    force = v ? atoi(v) : -1;
  }
  if (frank::num_sms() < 2 || force == 0) return false;
  return force == 1 || rows >= 1024 * E;
}

}  // namespace

namespace frank {

// Constraints checked here: K % 8 == 0 (16-byte TMA strides), N_out % 16 == 0,
// 16-byte aligned base pointers, rows and E*N within int32 coordinates.
int check_tc_shapes(int64_t rows, int64_t N, int64_t K, int64_t E) {
  if (K % 8 != 0 || K <= 0) {
    set_error("bf16 tensor-core path needs n_in %% 8 == 0 (got %lld)", (long long)K);
    return FRANK_EINVAL;
  }
  if (N % 16 != 0 || N <= 0) {
    set_error("bf16 tensor-core path needs n_out %% 16 == 0 (got %lld)", (long long)N);
    return FRANK_EINVAL;
  }
  if (E > kMaxExperts || rows > 0x7fffffffLL || N > 0x7fffffffLL) {
    set_error("bf16 tensor-core path: E=%lld rows=%lld N=%lld out of range", (long long)E, (long long)rows,
              (long long)N);
    return FRANK_EINVAL;
  }
  return FRANK_OK;
}

// mode: 0 SWIGLU (B = gate, B2 = up, out bf16 [rows, N]), 1 SCALE, 2 PLAIN
// (out fp32 [rows, N]).  A: bf16 [rows, K]; B/B2: bf16 [E, N, K].
int launch_tc_grouped_gemm(int mode, const void* A, const void* B, const void* B2, const int32_t* offsets, int64_t E,
                           int64_t rows, int64_t N, int64_t K, const float* wrow, void* out, cudaStream_t st,
                           const int32_t* row_rank, const int32_t* row_pos, float* const* peer_out, int n_peers,
                           int64_t peer_rows) {
  if (rows == 0) return FRANK_OK;
  FRANK_TRY(check_tc_shapes(rows, N, K, E));
  if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)(B2 ? B2 : B) | (uintptr_t)out) % 16 != 0) {
    set_error("bf16 tensor-core path needs 16-byte aligned buffers");
    return FRANK_EINVAL;
  }
  CUtensorMap ma, mb, mb2, ma16, ma32, ma64;
  FRANK_TRY(make_map_2d(&ma, A, rows, K));
  FRANK_TRY(make_map_2d(&ma16, A, rows, K, 16));
  FRANK_TRY(make_map_2d(&ma32, A, rows, K, 32));
  FRANK_TRY(make_map_2d(&ma64, A, rows, K, 64));
  FRANK_TRY(make_map_3d(&mb, B, E, N, K));
  if (mode == SWIGLU) FRANK_TRY(make_map_3d(&mb2, B2, E, N, K));
  else mb2 = mb;
  Params p;
  if (offsets == nullptr && E != 1) {
    set_error("tc_grouped_gemm: row offsets may be omitted only for a single group");
    return FRANK_EINVAL;
  }
  p.offsets = offsets;
  p.E = (int)E;
  p.rows = (int)rows;
  p.n_tiles = (int)(mode == SWIGLU ? (N + 127) / 128 : (N + BN - 1) / BN);
  p.N_out = (int)N;
  p.K = (int)K;
  p.out = out;
  p.ldo = N;
  p.wrow = wrow;
  p.err = device_error_word();
  p.row_rank = row_rank;
  p.row_pos = row_pos;
  for (int i = 0; i < kMaxPeers; ++i) p.peer_out[i] = (peer_out && i < n_peers) ? peer_out[i] : nullptr;
  p.n_peers = row_rank ? n_peers : 0;
  {
    // rows per band: a multiple of 256 (both tile heights) whose A rows fit
    // the L2 budget, at most 8192 (gate/up at K = 4096: 8192 rows, one band
    // per Mixtral expert; down at K = 14336: 2304 rows)
    int64_t br = kBandBytes / (K * 2);
    br = br / 256 * 256;
    p.band_rows = (int)(br < 256 ? 256 : (br > 8192 ? 8192 : br));
  }
  p.peer_rows = peer_rows;
  {
    const char* sw = getenv("FRANK_TC_SWAP");
    p.swap_small = (sw && sw[0] == '0') ? 0 : 1;
  }
  if (row_rank && (mode != SCALE || !row_pos || !peer_out || n_peers < 1 || n_peers > kMaxPeers)) {
    set_error("tc_grouped_gemm: a row map needs SCALE mode, row_pos and 1..%d peer buffers", kMaxPeers);
    return FRANK_EINVAL;
  }
  if (use_cta_pair(rows, E)) {
    size_t smem2 = smem2_bytes((int)E);
    dim3 grid2(num_sms() & ~1), block2(THREADS);
#define FRANK_TC2_CASE(M)                                                                                      \
  FRANK_CUDA_TRY(                                                                                              \
      cudaFuncSetAttribute(tc2_grouped_gemm_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2)); \
  tc2_grouped_gemm_kernel<M><<<grid2, block2, smem2, st>>>(ma, mb, mb2, p);
    switch (mode) {
      case SWIGLU: FRANK_TC2_CASE(SWIGLU) break;
      case SCALE: FRANK_TC2_CASE(SCALE) break;
      default: FRANK_TC2_CASE(PLAIN)
    }
#undef FRANK_TC2_CASE
    FRANK_LAUNCH_CHECK();
    return FRANK_OK;
  }
  size_t smem = smem_bytes((int)E);
  dim3 grid(num_sms()), block(THREADS);
  switch (mode) {
    case SWIGLU:
      FRANK_CUDA_TRY(cudaFuncSetAttribute(tc_grouped_gemm_kernel<SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
      tc_grouped_gemm_kernel<SWIGLU><<<grid, block, smem, st>>>(ma, mb, mb2, ma16, ma32, ma64, p);
      break;
    case SCALE:
      FRANK_CUDA_TRY(cudaFuncSetAttribute(tc_grouped_gemm_kernel<SCALE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
      tc_grouped_gemm_kernel<SCALE><<<grid, block, smem, st>>>(ma, mb, mb2, ma16, ma32, ma64, p);
      break;
    default:
      FRANK_CUDA_TRY(cudaFuncSetAttribute(tc_grouped_gemm_kernel<PLAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem));
      tc_grouped_gemm_kernel<PLAIN><<<grid, block, smem, st>>>(ma, mb, mb2, ma16, ma32, ma64, p);
  }
  FRANK_LAUNCH_CHECK();
  return FRANK_OK;
}

}  // namespace frank
