// C-ABI entry points (include/frank_moe.h) and the orchestration of the MoE
// FFN block / mul_mat_id out of the kernels in routing.cu, elementwise.cu,
// gemm_simt.cu and gemm_tc.cu.
#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace frank {

// ---- kernels implemented in the other translation units ----
int launch_softmax_topk(const float*, int64_t, int64_t, int64_t, int, float*, int32_t*, cudaStream_t);
int launch_router_topk(int, const void*, int, const void*, int64_t, int64_t, int64_t, int64_t, int, float*, int32_t*,
                       float*, cudaStream_t, const __nv_bfloat16* wr3_pre = nullptr);
size_t router_pack_offset(int64_t, int64_t);
size_t router_pack_bytes(int64_t, int64_t);
int launch_router_pack(int, const void*, int64_t, int64_t, void*, cudaStream_t);
size_t router_scratch_bytes(int, int64_t, int64_t, int64_t);
size_t permute_workspace_size(int64_t, int64_t);
int launch_permute(const int32_t*, int64_t, int64_t, int32_t*, int32_t*, int32_t*, int32_t*, void*, size_t,
                   cudaStream_t, const float* = nullptr, float* = nullptr);
int launch_swiglu(int, const void*, const void*, void*, int64_t, cudaStream_t);
int launch_prepack(int, const void*, int64_t, int64_t, int64_t, int, void*, cudaStream_t);
int launch_gather_rows(int, const void*, const int32_t*, int64_t, int64_t, int64_t, void*, cudaStream_t);
int launch_gather_cols(int, const void*, const int32_t*, int64_t, int64_t, void*, cudaStream_t,
                       const int32_t* = nullptr);
int launch_scatter_out(const float*, const int32_t*, int64_t, int64_t, float*, cudaStream_t);
int launch_combine(int, const float*, const int32_t*, int64_t, int64_t, int64_t, void*, cudaStream_t,
                   const float* residual = nullptr);
int launch_rms_norm(const float*, const float*, int64_t, int64_t, float, int, void*, cudaStream_t);
int launch_sorted_weights(const float*, const int32_t*, int64_t, float*, cudaStream_t);
int launch_copy_row_segments(const void*, void*, const int64_t*, const int64_t*, const int64_t*, int64_t, int64_t,
                             int64_t, cudaStream_t);
int launch_grouped_gemm_f32(int, const float*, const float*, const float*, const int32_t*, int64_t, int64_t, int64_t,
                            int64_t, const float*, float*, cudaStream_t);
int launch_tc_grouped_gemm(int, const void*, const void*, const void*, const int32_t*, int64_t, int64_t, int64_t,
                           int64_t, const float*, void*, cudaStream_t, const int32_t* row_rank = nullptr,
                           const int32_t* row_pos = nullptr, float* const* peer_out = nullptr, int n_peers = 0,
                           int64_t peer_rows = 0);
int check_tc_shapes(int64_t, int64_t, int64_t, int64_t);
bool decode_path_ok(int, int64_t, int64_t, int64_t, int64_t, int64_t);
size_t decode_workspace_size(int64_t, int64_t, int64_t, int64_t, int64_t);
int launch_decode_block(const void*, int, const void*, const void*, const void*, const void*, int64_t, int64_t,
                        int64_t, int64_t, int64_t, int, int, void*, float*, int32_t*, void*, size_t, cudaStream_t,
                        void (*)(int, cudaStream_t), const float* residual);

// ---- error state ----
static thread_local std::string g_err;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
}

__device__ int32_t g_device_error = 0;

static std::atomic<uint64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// Stage timing (frank_profile_stages / frank_profile_read): one set of
// events per profiled call, kept for up to kProfCalls calls; reading
// averages over the recorded calls and starts a new window.
constexpr int kStages = 6;
constexpr int kProfCalls = 64;
struct StageProfiler {
  bool on = false;
  bool fixed = false;  // graph-capture mode: always the first event set, kept across reads
  bool init = false;
  int calls = 0;    // calls recorded in the current window
  int marks = 0;    // marks recorded in the current call
  cudaEvent_t ev[kProfCalls][kStages + 1];
};
static StageProfiler g_prof;
static std::mutex g_prof_mu;

static void prof_mark(int i, cudaStream_t st) {
  if (!g_prof.on) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  if (!g_prof.init) {
    for (auto& set : g_prof.ev)
      for (auto& e : set) cudaEventCreate(&e);
    g_prof.init = true;
  }
  if (g_prof.fixed) {
    // external record nodes: a captured graph records the event on each replay
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs == cudaStreamCaptureStatusActive)
      cudaEventRecordWithFlags(g_prof.ev[0][i], st, cudaEventRecordExternal);
    else
      cudaEventRecord(g_prof.ev[0][i], st);
    if (i == kStages) g_prof.calls = 1;
    return;
  }
  if (g_prof.calls >= kProfCalls) return;
  cudaEventRecord(g_prof.ev[g_prof.calls][i], st);
  if (i == kStages) ++g_prof.calls;
}

int32_t* device_error_word() {
  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static std::vector<int32_t*> cache;
  std::lock_guard<std::mutex> lk(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, nullptr);
  if (!cache[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<int32_t*>(p);
  }
  return cache[dev];
}

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static std::vector<int> cache;
  std::lock_guard<std::mutex> lk(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 1;
  }
  return cache[dev];
}

// ---- workspace layouts ----
struct MoeWs {
  float* w;
  int32_t* ids;
  int32_t* sorted_slots;
  int32_t* offsets;
  int32_t* slot_pos;
  int32_t* err;
  float* wsorted;
  void* xs;
  void* hs;
  float* ds;
  float* logits;
  void* perm_ws;
  size_t perm_bytes;
};

static size_t moe_layout(int dtype, int64_t T, int64_t H, int64_t F, int64_t E, int64_t k, void* base, size_t cap,
                         MoeWs* L) {
  const int64_t n = k * T;
  const size_t esz = dtype == FRANK_F32 ? 4 : 2;
  Carve c(base, cap);
  MoeWs l;
  c.take<char>(1);  // the workspace header (the decode kernel's counters; untouched here)
  l.w = c.take<float>(n);
  l.ids = c.take<int32_t>(n);
  l.sorted_slots = c.take<int32_t>(n);
  l.offsets = c.take<int32_t>(E + 1);
  l.slot_pos = c.take<int32_t>(n);
  l.err = c.take<int32_t>(1);
  l.wsorted = c.take<float>(n);
  l.xs = c.take<char>(n * H * esz);
  l.hs = c.take<char>(n * F * esz);
  l.ds = c.take<float>(n * H);
  l.logits = c.take<float>(router_scratch_bytes(dtype, T, H, E) / sizeof(float) + 1);
  l.perm_bytes = permute_workspace_size(n, E);
  l.perm_ws = c.take<char>(l.perm_bytes);
  if (L) *L = l;
  return align_up(c.used, 256);
}

struct MmidWs {
  int32_t* sorted_slots;
  int32_t* offsets;
  int32_t* slot_pos;
  void* xs;
  float* ys;
  void* perm_ws;
  size_t perm_bytes;
};

static size_t mmid_layout(int dtype, int64_t O, int64_t I, int64_t E, int64_t k, int64_t T, void* base, size_t cap,
                          MmidWs* L) {
  const int64_t n = k * T;
  const size_t esz = dtype == FRANK_F32 ? 4 : 2;
  Carve c(base, cap);
  MmidWs l;
  l.sorted_slots = c.take<int32_t>(n);
  l.offsets = c.take<int32_t>(E + 1);
  l.slot_pos = c.take<int32_t>(n);
  l.xs = c.take<char>(n * I * esz);
  l.ys = c.take<float>(n * O);
  l.perm_bytes = permute_workspace_size(n, E);
  l.perm_ws = c.take<char>(l.perm_bytes);
  if (L) *L = l;
  return align_up(c.used, 256);
}

// A router pack (FRANK_ROUTER_PACKED) is an fp32 wr followed by its bf16
// split: every path reads the fp32 part, the tensor-core router the split.
static const __nv_bfloat16* resolve_router(int* wr_dtype, const void* wr, int64_t E, int64_t H) {
  if (*wr_dtype != FRANK_ROUTER_PACKED) return nullptr;
  *wr_dtype = FRANK_F32;
  return reinterpret_cast<const __nv_bfloat16*>(static_cast<const char*>(wr) + router_pack_offset(E, H));
}

static int check_dtype(int d, const char* what) {
  if (d != FRANK_F32 && d != FRANK_BF16) {
    set_error("%s: dtype %d is neither FRANK_F32 (0) nor FRANK_BF16 (1)", what, d);
    return FRANK_EINVAL;
  }
  return FRANK_OK;
}

}  // namespace frank

using namespace frank;

extern "C" {

const char* frank_last_error(void) { return g_err.c_str(); }

int frank_abi_version(void) { return 102; }

int frank_num_sms(void) { return num_sms(); }

int frank_swiglu(int dtype, const void* gate, const void* up, void* out, int64_t n, void* stream) {
  FRANK_TRY(check_dtype(dtype, "swiglu"));
  FRANK_CHECK_ARG(n >= 0, "swiglu: n=%lld < 0", (long long)n);
  FRANK_CHECK_ARG(n == 0 || (gate && up && out), "swiglu: null pointer");
  return launch_swiglu(dtype, gate, up, out, n, as_stream(stream));
}

int frank_softmax_topk(const float* logits, int64_t T, int64_t E, int64_t k, int normalize, float* weights,
                       int32_t* ids, void* stream) {
  FRANK_CHECK_ARG(E >= 1 && E <= 256, "softmax_topk: E=%lld outside [1, 256]", (long long)E);
  FRANK_CHECK_ARG(k >= 1 && k <= E && k <= 32, "softmax_topk: k=%lld outside [1, min(E, 32)]", (long long)k);
  FRANK_CHECK_ARG(T >= 0, "softmax_topk: T < 0");
  return launch_softmax_topk(logits, T, E, k, normalize, weights, ids, as_stream(stream));
}

size_t frank_router_scratch_bytes(int x_dtype, int64_t T, int64_t H, int64_t E) {
  return router_scratch_bytes(x_dtype, T, H, E);
}

int frank_router_topk(int x_dtype, const void* x, int wr_dtype, const void* wr, int64_t T, int64_t H, int64_t E,
                      int64_t k, int normalize, float* weights, int32_t* ids, float* logits_scratch, void* stream) {
  FRANK_TRY(check_dtype(x_dtype, "router_topk"));
  const __nv_bfloat16* wr3 = resolve_router(&wr_dtype, wr, E, H);
  FRANK_TRY(check_dtype(wr_dtype, "router_topk"));
  FRANK_CHECK_ARG(E >= 1 && E <= 256, "router_topk: E=%lld outside [1, 256]", (long long)E);
  FRANK_CHECK_ARG(k >= 1 && k <= E && k <= 32, "router_topk: k=%lld outside [1, min(E, 32)]", (long long)k);
  FRANK_CHECK_ARG(T >= 0 && H >= 1, "router_topk: bad T=%lld / H=%lld", (long long)T, (long long)H);
  return launch_router_topk(x_dtype, x, wr_dtype, wr, T, H, E, k, normalize, weights, ids, logits_scratch,
                            as_stream(stream), wr3);
}

size_t frank_router_pack_size(int64_t E, int64_t H) { return router_pack_bytes(E, H); }
size_t frank_router_pack_offset(int64_t E, int64_t H) { return router_pack_offset(E, H); }

int frank_router_pack(int wr_dtype, const void* wr, int64_t E, int64_t H, void* pack, void* stream) {
  FRANK_TRY(check_dtype(wr_dtype, "router_pack"));
  FRANK_CHECK_ARG(E >= 1 && E <= 256 && H >= 1, "router_pack: bad E=%lld / H=%lld", (long long)E, (long long)H);
  FRANK_CHECK_ARG(wr && pack && (uintptr_t)pack % 256 == 0, "router_pack: null or unaligned pointer");
  return launch_router_pack(wr_dtype, wr, E, H, pack, as_stream(stream));
}

size_t frank_permute_workspace_size(int64_t n_slots, int64_t E) { return permute_workspace_size(n_slots, E); }

int frank_permute(const int32_t* ids, int64_t n_slots, int64_t E, int32_t* sorted_slots, int32_t* offsets,
                  int32_t* slot_pos, int32_t* err_flag, void* workspace, size_t ws_bytes, void* stream) {
  FRANK_CHECK_ARG(n_slots >= 0 && n_slots < 0x7fffffffLL, "permute: n_slots=%lld out of range", (long long)n_slots);
  return launch_permute(ids, n_slots, E, sorted_slots, offsets, slot_pos, err_flag, workspace, ws_bytes,
                        as_stream(stream));
}

int frank_prepack_experts(int in_dtype, const void* w_oie, int64_t O, int64_t I, int64_t E, int out_dtype,
                          void* w_eoi, void* stream) {
  FRANK_TRY(check_dtype(in_dtype, "prepack"));
  FRANK_TRY(check_dtype(out_dtype, "prepack"));
  FRANK_CHECK_ARG(O >= 0 && I >= 0 && E >= 0, "prepack: negative extent");
  return launch_prepack(in_dtype, w_oie, O, I, E, out_dtype, w_eoi, as_stream(stream));
}

size_t frank_mul_mat_id_workspace_size(int dtype, int64_t O, int64_t I, int64_t E, int64_t k, int64_t T) {
  return mmid_layout(dtype, O, I, E, k, T, nullptr, 0, nullptr);
}

int frank_mul_mat_id(int dtype, const void* w_eoi, const void* input, const int32_t* ids, int64_t O, int64_t I,
                     int64_t E, int64_t k, int64_t T, float* out, int32_t* err_flag, void* workspace,
                     size_t ws_bytes, void* stream) {
  FRANK_TRY(check_dtype(dtype, "mul_mat_id"));
  FRANK_CHECK_ARG(O >= 1 && I >= 1 && E >= 1 && k >= 1 && T >= 0, "mul_mat_id: bad shape O=%lld I=%lld E=%lld k=%lld T=%lld",
                  (long long)O, (long long)I, (long long)E, (long long)k, (long long)T);
  cudaStream_t st = as_stream(stream);
  const int64_t n = k * T;
  if (n == 0) return FRANK_OK;
  if (dtype == FRANK_BF16) FRANK_TRY(check_tc_shapes(n, O, I, E));
  size_t need = mmid_layout(dtype, O, I, E, k, T, nullptr, 0, nullptr);
  if (ws_bytes < need) {
    set_error("mul_mat_id: workspace %zu < %zu bytes", ws_bytes, need);
    return FRANK_ENOSPC;
  }
  MmidWs L;
  mmid_layout(dtype, O, I, E, k, T, workspace, ws_bytes, &L);
  FRANK_TRY(launch_permute(ids, n, E, L.sorted_slots, L.offsets, L.slot_pos, err_flag, L.perm_ws, L.perm_bytes, st));
  FRANK_TRY(launch_gather_cols(dtype, input, L.sorted_slots, n, I, L.xs, st, L.slot_pos));
  if (dtype == FRANK_F32) {
    FRANK_TRY(launch_grouped_gemm_f32(0, (const float*)L.xs, (const float*)w_eoi, nullptr, L.offsets, E, n, O, I,
                                      nullptr, L.ys, st));
  } else {
    FRANK_TRY(launch_tc_grouped_gemm(2, L.xs, w_eoi, nullptr, L.offsets, E, n, O, I, nullptr, L.ys, st));
  }
  return launch_scatter_out(L.ys, L.slot_pos, n, O, out, st);
}

size_t frank_moe_ffn_block_workspace_size(int dtype, int64_t T, int64_t H, int64_t F, int64_t E, int64_t k) {
  if (decode_path_ok(dtype, T, H, F, E, k)) return decode_workspace_size(T, H, F, E, k);
  return moe_layout(dtype, T, H, F, E, k, nullptr, 0, nullptr);
}

namespace {

// The block (see frank_moe_ffn_block); residual: optional fp32 [T, H] added
// to y after the sum over the k slots (the sub-layer's residual connection).
int moe_block(int dtype, const void* x, int wr_dtype, const void* wr, const void* w_up_p, const void* w_gate_p,
              const void* w_down_p, int64_t T, int64_t E, int64_t k, int64_t H, int64_t F, int normalize, int y_dtype,
              void* y, float* route_w, int32_t* route_ids, void* workspace, size_t ws_bytes, cudaStream_t st,
              const float* residual) {
  FRANK_TRY(check_dtype(dtype, "moe_ffn_block"));
  const __nv_bfloat16* wr3 = resolve_router(&wr_dtype, wr, E, H);
  FRANK_TRY(check_dtype(wr_dtype, "moe_ffn_block"));
  FRANK_TRY(check_dtype(y_dtype, "moe_ffn_block"));
  FRANK_CHECK_ARG(E >= 1 && E <= 256, "moe_ffn_block: n_expert=%lld outside [1, 256]", (long long)E);
  FRANK_CHECK_ARG(k >= 1 && k <= E && k <= 32, "moe_ffn_block: n_expert_used=%lld outside [1, min(E, 32)]",
                  (long long)k);
  FRANK_CHECK_ARG(T >= 0 && H >= 1 && F >= 1, "moe_ffn_block: bad T=%lld H=%lld F=%lld", (long long)T, (long long)H,
                  (long long)F);
  if (T == 0) return FRANK_OK;
  const int64_t n = k * T;
  if (dtype == FRANK_BF16) {
    FRANK_TRY(check_tc_shapes(n, F, H, E));
    FRANK_TRY(check_tc_shapes(n, H, F, E));
    FRANK_CHECK_ARG(H % 4 == 0, "moe_ffn_block bf16: n_embd %% 4 != 0");
  }
  if (decode_path_ok(dtype, T, H, F, E, k)) {
    // a few tokens: weight-streaming decode kernels (csrc/decode.cu)
    return launch_decode_block(x, wr_dtype, wr, w_up_p, w_gate_p, w_down_p, T, E, k, H, F, normalize, y_dtype, y,
                               route_w, route_ids, workspace, ws_bytes, st, prof_mark, residual);
  }
  size_t need = moe_layout(dtype, T, H, F, E, k, nullptr, 0, nullptr);
  if (ws_bytes < need) {
    set_error("moe_ffn_block: workspace %zu < %zu bytes", ws_bytes, need);
    return FRANK_ENOSPC;
  }
  MoeWs L;
  moe_layout(dtype, T, H, F, E, k, workspace, ws_bytes, &L);
  float* w = route_w ? route_w : L.w;
  int32_t* ids = route_ids ? route_ids : L.ids;
  prof_mark(0, st);
  // 1. router + softmax + top-k (+ renorm)          moe_ffn_block.mlir:54-128
  FRANK_TRY(launch_router_topk(dtype, x, wr_dtype, wr, T, H, E, k, normalize, w, ids, L.logits, st, wr3));
  prof_mark(1, st);
  // 2. stable expert permutation                    mul_mat_id.mlir:51-61
  FRANK_TRY(launch_permute(ids, n, E, L.sorted_slots, L.offsets, L.slot_pos, nullptr, L.perm_ws, L.perm_bytes, st,
                           w, L.wsorted));
  prof_mark(2, st);
  // 3. expert-sorted activation rows (replicate + permute, :130-144, mul_mat_id.mlir:64-84)
  FRANK_TRY(launch_gather_rows(dtype, x, L.sorted_slots, n, T, H, L.xs, st));
  prof_mark(3, st);
  if (dtype == FRANK_F32) {
    // 4. h = gate(x) * silu(up(x))                   :146-156
    FRANK_TRY(launch_grouped_gemm_f32(2, (const float*)L.xs, (const float*)w_gate_p, (const float*)w_up_p, L.offsets,
                                      E, n, F, H, nullptr, (float*)L.hs, st));
    prof_mark(4, st);
    // 5. d = down(h) * w                             :158-177
    FRANK_TRY(launch_grouped_gemm_f32(1, (const float*)L.hs, (const float*)w_down_p, nullptr, L.offsets, E, n, H, F,
                                      L.wsorted, L.ds, st));
  } else {
    FRANK_TRY(launch_tc_grouped_gemm(0, L.xs, w_gate_p, w_up_p, L.offsets, E, n, F, H, nullptr, L.hs, st));
    prof_mark(4, st);
    FRANK_TRY(launch_tc_grouped_gemm(1, L.hs, w_down_p, nullptr, L.offsets, E, n, H, F, L.wsorted, L.ds, st));
  }
  prof_mark(5, st);
  // 6. y[t] = sum_j d[slot j of t]                   :179-206
  FRANK_TRY(launch_combine(y_dtype, L.ds, L.slot_pos, T, k, H, y, st, residual));
  prof_mark(6, st);
  return FRANK_OK;
}

}  // namespace

int frank_moe_ffn_block(int dtype, const void* x, int wr_dtype, const void* wr, const void* w_up_p,
                        const void* w_gate_p, const void* w_down_p, int64_t T, int64_t E, int64_t k, int64_t H,
                        int64_t F, int normalize, int y_dtype, void* y, float* route_w, int32_t* route_ids, void* workspace,
                        size_t ws_bytes, void* stream) {
  return moe_block(dtype, x, wr_dtype, wr, w_up_p, w_gate_p, w_down_p, T, E, k, H, F, normalize, y_dtype, y, route_w,
                   route_ids, workspace, ws_bytes, as_stream(stream), nullptr);
}

int frank_rms_norm(const float* x, const float* weight, int64_t T, int64_t H, float eps, int out_dtype, void* out,
                   void* stream) {
  FRANK_TRY(check_dtype(out_dtype, "rms_norm"));
  FRANK_CHECK_ARG(T >= 0 && H >= 1, "rms_norm: bad T=%lld H=%lld", (long long)T, (long long)H);
  FRANK_CHECK_ARG(T == 0 || (x && weight && out), "rms_norm: null pointer");
  return launch_rms_norm(x, weight, T, H, eps, out_dtype, out, as_stream(stream));
}

size_t frank_moe_ffn_sublayer_workspace_size(int dtype, int64_t T, int64_t H, int64_t F, int64_t E, int64_t k) {
  return align_up((size_t)T * H * (dtype == FRANK_F32 ? 4 : 2), 256) +
         frank_moe_ffn_block_workspace_size(dtype, T, H, F, E, k);
}

int frank_moe_ffn_sublayer(int dtype, const float* residual, const float* norm_w, float eps, int wr_dtype,
                           const void* wr, const void* w_up_p, const void* w_gate_p, const void* w_down_p, int64_t T,
                           int64_t E, int64_t k, int64_t H, int64_t F, int normalize, float* out, float* route_w,
                           int32_t* route_ids, void* workspace, size_t ws_bytes, void* stream) {
  FRANK_TRY(check_dtype(dtype, "moe_ffn_sublayer"));
  FRANK_CHECK_ARG(T >= 0 && H >= 1, "moe_ffn_sublayer: bad T=%lld H=%lld", (long long)T, (long long)H);
  if (T == 0) return FRANK_OK;
  FRANK_CHECK_ARG(residual && norm_w && out, "moe_ffn_sublayer: null pointer");
  const size_t need = frank_moe_ffn_sublayer_workspace_size(dtype, T, H, F, E, k);
  if (ws_bytes < need) {
    set_error("moe_ffn_sublayer: workspace %zu < %zu bytes", ws_bytes, need);
    return FRANK_ENOSPC;
  }
  cudaStream_t st = as_stream(stream);
  // the block's workspace first (its header stays at offset 0 for every T),
  // the normalised tokens after it
  const size_t blk_bytes = frank_moe_ffn_block_workspace_size(dtype, T, H, F, E, k);
  void* xn = static_cast<char*>(workspace) + blk_bytes;
  FRANK_TRY(launch_rms_norm(residual, norm_w, T, H, eps, dtype, xn, st));
  return moe_block(dtype, xn, wr_dtype, wr, w_up_p, w_gate_p, w_down_p, T, E, k, H, F, normalize, FRANK_F32, out,
                   route_w, route_ids, workspace, blk_bytes, st, residual);
}

int frank_gather_rows(int dtype, const void* x, const int32_t* sorted_slots, int64_t rows, int64_t T, int64_t H,
                      void* xs, void* stream) {
  FRANK_TRY(check_dtype(dtype, "gather_rows"));
  FRANK_CHECK_ARG(rows >= 0 && T >= 1 && H >= 1, "gather_rows: bad rows/T/H");
  return launch_gather_rows(dtype, x, sorted_slots, rows, T, H, xs, as_stream(stream));
}

int frank_gather_weights(const float* w, const int32_t* sorted_slots, int64_t n, float* w_sorted, void* stream) {
  FRANK_CHECK_ARG(n >= 0, "gather_weights: n < 0");
  return launch_sorted_weights(w, sorted_slots, n, w_sorted, as_stream(stream));
}

size_t frank_expert_ffn_workspace_size(int dtype, int64_t rows, int64_t F) {
  return align_up((size_t)rows * F * (dtype == FRANK_F32 ? 4 : 2), 256) + 256;
}

int frank_expert_ffn(int dtype, const void* xs, const float* w_rows, const int32_t* offsets, int64_t E, int64_t rows,
                     int64_t H, int64_t F, const void* w_up_p, const void* w_gate_p, const void* w_down_p, float* d,
                     void* workspace, size_t ws_bytes, void* stream) {
  FRANK_TRY(check_dtype(dtype, "expert_ffn"));
  FRANK_CHECK_ARG(E >= 1 && rows >= 0 && H >= 1 && F >= 1, "expert_ffn: bad shape");
  if (rows == 0) return FRANK_OK;
  if (ws_bytes < frank_expert_ffn_workspace_size(dtype, rows, F)) {
    set_error("expert_ffn: workspace %zu < %zu bytes", ws_bytes, frank_expert_ffn_workspace_size(dtype, rows, F));
    return FRANK_ENOSPC;
  }
  cudaStream_t st = as_stream(stream);
  if (dtype == FRANK_F32) {
    FRANK_TRY(launch_grouped_gemm_f32(2, (const float*)xs, (const float*)w_gate_p, (const float*)w_up_p, offsets, E,
                                      rows, F, H, nullptr, (float*)workspace, st));
    return launch_grouped_gemm_f32(1, (const float*)workspace, (const float*)w_down_p, nullptr, offsets, E, rows, H,
                                   F, w_rows, d, st);
  }
  FRANK_TRY(check_tc_shapes(rows, F, H, E));
  FRANK_TRY(check_tc_shapes(rows, H, F, E));
  FRANK_TRY(launch_tc_grouped_gemm(0, xs, w_gate_p, w_up_p, offsets, E, rows, F, H, nullptr, workspace, st));
  return launch_tc_grouped_gemm(1, workspace, w_down_p, nullptr, offsets, E, rows, H, F, w_rows, d, st);
}

int frank_expert_ffn_scatter(const void* xs, const float* w_rows, const int32_t* offsets, int64_t E, int64_t rows,
                             int64_t H, int64_t F, const void* w_up_p, const void* w_gate_p, const void* w_down_p,
                             const int32_t* row_rank, const int32_t* row_pos, void* const* peer_out, int n_peers,
                             int64_t peer_rows, void* workspace, size_t ws_bytes, void* stream) {
  FRANK_CHECK_ARG(E >= 1 && rows >= 0 && H >= 1 && F >= 1, "expert_ffn_scatter: bad shape");
  FRANK_CHECK_ARG(row_rank && row_pos && peer_out && n_peers >= 1 && peer_rows >= 0,
                  "expert_ffn_scatter: missing row map / peers");
  if (rows == 0) return FRANK_OK;
  if (ws_bytes < frank_expert_ffn_workspace_size(FRANK_BF16, rows, F)) {
    set_error("expert_ffn_scatter: workspace %zu < %zu bytes", ws_bytes,
              frank_expert_ffn_workspace_size(FRANK_BF16, rows, F));
    return FRANK_ENOSPC;
  }
  cudaStream_t st = as_stream(stream);
  FRANK_TRY(check_tc_shapes(rows, F, H, E));
  FRANK_TRY(check_tc_shapes(rows, H, F, E));
  FRANK_TRY(launch_tc_grouped_gemm(0, xs, w_gate_p, w_up_p, offsets, E, rows, F, H, nullptr, workspace, st));
  return launch_tc_grouped_gemm(1, workspace, w_down_p, nullptr, offsets, E, rows, H, F, w_rows, nullptr, st,
                                row_rank, row_pos, reinterpret_cast<float* const*>(peer_out), n_peers, peer_rows);
}

int frank_combine(const float* d, const int32_t* slot_pos, int64_t T, int64_t k, int64_t H, int y_dtype, void* y,
                  void* stream) {
  FRANK_TRY(check_dtype(y_dtype, "combine"));
  FRANK_CHECK_ARG(T >= 0 && k >= 1 && H >= 1, "combine: bad shape");
  return launch_combine(y_dtype, d, slot_pos, T, k, H, y, as_stream(stream));
}

int frank_copy_row_segments(const void* src, void* dst, const int64_t* src_start, const int64_t* dst_start,
                            const int64_t* seg_prefix, int64_t nseg, int64_t total_rows, int64_t row_bytes,
                            void* stream) {
  FRANK_CHECK_ARG(nseg >= 0 && total_rows >= 0 && row_bytes > 0, "copy_row_segments: bad arguments");
  return launch_copy_row_segments(src, dst, src_start, dst_start, seg_prefix, nseg, total_rows, row_bytes,
                                  as_stream(stream));
}

int frank_read_device_error(int32_t* out, void* stream) {
  int32_t* p = device_error_word();
  if (!p) {
    set_error("device error word unavailable");
    return FRANK_ECUDA;
  }
  cudaStream_t st = as_stream(stream);
  int32_t v = 0;
  FRANK_CUDA_TRY(cudaMemcpyAsync(&v, p, sizeof(v), cudaMemcpyDeviceToHost, st));
  FRANK_CUDA_TRY(cudaMemsetAsync(p, 0, sizeof(v), st));
  FRANK_CUDA_TRY(cudaStreamSynchronize(st));
  if (out) *out = v;
  return FRANK_OK;
}

uint64_t frank_launch_count(void) { return g_launches.load(); }

int frank_profile_stages(int enable) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof.on = enable != 0;
  if (enable) {  // disabling keeps the mode so recorded events can still be read
    g_prof.fixed = enable == 2;
    g_prof.calls = 0;
  }
  return FRANK_OK;
}

int frank_profile_read(float* stage_ms, int max_stages, int* n_stages) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  if (!g_prof.init || g_prof.calls == 0) {
    set_error("profile_read: no complete profiled call recorded");
    return FRANK_EINVAL;
  }
  const int n = max_stages < kStages ? max_stages : kStages;
  FRANK_CUDA_TRY(cudaEventSynchronize(g_prof.ev[g_prof.calls - 1][kStages]));
  for (int i = 0; i < n; ++i) {
    double acc = 0.0;
    for (int c = 0; c < g_prof.calls; ++c) {
      float ms = 0.f;
      FRANK_CUDA_TRY(cudaEventElapsedTime(&ms, g_prof.ev[c][i], g_prof.ev[c][i + 1]));
      acc += ms;
    }
    stage_ms[i] = (float)(acc / g_prof.calls);
  }
  if (n_stages) *n_stages = g_prof.calls;
  if (!g_prof.fixed) g_prof.calls = 0;
  return FRANK_OK;
}

}  // extern "C"
