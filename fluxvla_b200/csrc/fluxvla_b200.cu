// C ABI of the fluxvla_b200 kernels (declared in include/fluxvla_b200.h).
// Host side: argument checks, TMA tensor-map encoding, grid sizing, launch.
// No entry point allocates, synchronises or exits.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "attention.cuh"
#include "attention_tc.cuh"
#include "common.cuh"
#include "elementwise.cuh"
#include "expert_mega.cuh"
#include "gemm_tc.cuh"
#include "gemm_pair.cuh"

namespace {

thread_local char g_err[512] = "";
std::atomic<long long> g_launches{0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(FVB_ERR_CUDA, "%s: launch failed: %s", what,
                cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return FVB_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t,
                                  void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p,
                                cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D bf16 tensor map over [rows, k] (row stride ld elements), box
// [box_rows, 64] with the 128-byte swizzle; out-of-range reads fill zeros.
int make_map(CUtensorMap* m, const void* ptr, int64_t rows, int64_t k,
             int64_t ld, int box_rows) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return fail(FVB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FVB_ERR_INVALID_ARG, "tensor map encode failed (%d)", (int)r);
  return FVB_OK;
}

// Output tensor map of a normal-orientation GEMM epilogue: [rows, cols] of
// f32 or bf16 (row stride ld elements), box [32, box_cols] with the swizzle
// whose span equals the box row (64 or 32 bytes).
int make_out_map(CUtensorMap* m, void* ptr, bool f32, int64_t rows,
                 int64_t cols, int64_t ld, int box_cols) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return fail(FVB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const int eb = f32 ? 4 : 2;
  const int row_bytes = box_cols * eb;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * eb)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                  : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult r = enc(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                          : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                   2, ptr, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FVB_ERR_INVALID_ARG, "output tensor map encode failed (%d)", (int)r);
  return FVB_OK;
}

// Output tensor map with a dense (unswizzled) box of box_rows x box_cols.
int make_out_map_dense(CUtensorMap* m, void* ptr, bool f32, int64_t rows,
                       int64_t cols, int64_t ld, int box_cols, int box_rows) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return fail(FVB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const int eb = f32 ? 4 : 2;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * eb)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                          : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                   2, ptr, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FVB_ERR_INVALID_ARG, "output tensor map encode failed (%d)", (int)r);
  return FVB_OK;
}

// Tensor map over a bf16 [layers, rows, dim] cache, box 64 x 64 x 1 with
// 128-byte swizzle (rows past `rows` read as zeros).
int make_cache_map(CUtensorMap* m, const void* ptr, int64_t layers, int64_t rows,
                   int64_t dim) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return fail(FVB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)dim, (cuuint64_t)rows, (cuuint64_t)layers};
  cuuint64_t strides[2] = {(cuuint64_t)dim * 2, (cuuint64_t)(rows * dim * 2)};
  cuuint32_t box[3] = {64, 64, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FVB_ERR_INVALID_ARG, "cache tensor map encode failed (%d)", (int)r);
  return FVB_OK;
}

// TMA-store epilogues are on unless FVB_TMA_OUT=0.
bool tma_out_enabled() {
  static const int v = [] {
    const char* e = getenv("FVB_TMA_OUT");
    return e ? atoi(e) : 1;
  }();
  return v != 0;
}

// Programmatic dependent launch is on unless FVB_PDL=0: each kernel may
// start its prologue (and the GEMMs their weight prefetch) while the
// previous kernel in the stream drains; every kernel executes
// griddepcontrol.wait before touching data produced upstream.
bool pdl_enabled() {
  static const int v = [] {
    const char* e = getenv("FVB_PDL");
    return e ? atoi(e) : 1;
  }();
  return v != 0;
}

template <typename... KArgs, typename... Args>
int launch_k(const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block,
             size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess)
    return fail(FVB_ERR_CUDA, "%s: launch failed: %s", what,
                cudaGetErrorString(e));
  return check_launch(what);
}

int sm_count() {
  static int counts[128] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 148;
  if (!counts[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = n > 0 ? n : 148;
  }
  return counts[dev];
}


// cudaFuncSetAttribute applies to the current device only, so the raised
// dynamic shared memory limit is remembered per (kernel, device): a process
// that drives several GPUs through this library sets it on each of them.
int ensure_smem(const void* kern, int bytes, const char* what) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(FVB_ERR_CUDA, "%s: cudaGetDevice: %s", what, cudaGetErrorString(e));
  std::lock_guard<std::mutex> lk(mu);
  if (done.count({kern, dev})) return FVB_OK;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    return fail(FVB_ERR_CUDA, "%s: shared memory attribute: %s", what,
                cudaGetErrorString(e));
  done.insert({kern, dev});
  return FVB_OK;
}

template <int BN, int EPI, bool SWAP, int ACT = FVB_ACT_NONE>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb,
                const CUtensorMap& mo, const fvb::GemmDev& d, cudaStream_t st) {
  using C = fvb::GemmCfg<BN>;
  auto kern = fvb::gemm_tc_kernel<BN, C::STAGES, EPI, SWAP, ACT>;
  if (int rr = ensure_smem(reinterpret_cast<const void*>(kern), C::SMEM, "gemm")) return rr;
  const int grid = d.n_work < sm_count() ? d.n_work : sm_count();
  return launch_k("fvb_gemm", kern, dim3(grid), dim3(fvb::GEMM_THREADS),
                  (size_t)C::SMEM, st, ma, mb, mo, d);
}

int g_trace_next = 0;

template <int BN, int EPI>
int launch_gemm_pair(const CUtensorMap& ma, const CUtensorMap& mb,
                     const CUtensorMap& mo, const fvb::GemmDev& d, cudaStream_t st) {
  using C = fvb::pair::PairCfg<BN>;
  auto kern = fvb::pair::gemm_pair_kernel<BN, EPI>;
  if (int rr = ensure_smem(reinterpret_cast<const void*>(kern), C::SMEM, "gemm pair")) return rr;
  const int pairs_max = sm_count() / 2;
  const int pairs = d.n_work < pairs_max ? d.n_work : pairs_max;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(fvb::pair::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 2;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ma, mb, mo, d);
  if (e != cudaSuccess)
    return fail(FVB_ERR_CUDA, "fvb_gemm (pair): launch failed: %s", cudaGetErrorString(e));
  return check_launch("fvb_gemm (pair)");
}

int gemm_pair(const fvb_gemm_args* a, void* stream) {
  constexpr int BN = 208;
  if (!a->swap || (a->epilogue != FVB_EPI_GEGLU && a->epilogue != FVB_EPI_F32_ACC) ||
      (a->block_n != 0 && a->block_n != BN) || a->norm_out || a->row_add)
    return fail(FVB_ERR_UNSUPPORTED,
                "fvb_gemm: pair tiles need swap, GEGLU or F32_ACC, block_n 208");
  if (a->epilogue == FVB_EPI_GEGLU && (a->m % 2 || a->ldo % 1))
    return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: GEGLU needs an even feature count");
  const int k_tiles = (a->k + fvb::GEMM_BK - 1) / fvb::GEMM_BK;
  int split = a->split_k > 0 ? a->split_k : 1;
  if (split > k_tiles) split = k_tiles;
  const int kt_per = (k_tiles + split - 1) / split;
  split = (k_tiles + kt_per - 1) / kt_per;
  if (split > 1 && a->epilogue != FVB_EPI_F32_ACC)
    return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: pair split-K needs FVB_EPI_F32_ACC");
  const bool geglu = a->epilogue == FVB_EPI_GEGLU;
  if ((reinterpret_cast<uintptr_t>(a->out) & 15) || (a->ldo * (geglu ? 2 : 4)) % 16)
    return fail(FVB_ERR_INVALID_ARG,
                "fvb_gemm: pair tiles need a 16-byte aligned output and row stride");
  CUtensorMap ma, mb, mo;
  int r = make_map(&ma, a->a, a->m, a->k, a->lda, 128);
  if (!r) r = make_map(&mb, a->b, a->n, a->k, a->ldb, BN / 2);
  if (!r) r = make_out_map_dense(&mo, a->out, !geglu, a->n, geglu ? a->m / 2 : a->m,
                                 a->ldo, geglu ? 16 : 32, 16);
  if (r) return r;
  fvb::GemmDev d;
  memset(&d, 0, sizeof(d));
  d.m = a->m; d.n = a->n; d.k = a->k;
  d.k_tiles = k_tiles; d.kt_per_split = kt_per; d.split = split;
  d.out = a->out; d.ldo = a->ldo;
  d.bias = a->bias; d.gate = a->gate; d.alpha = a->alpha;
  d.m_tiles = (a->m + 255) / 256;
  d.n_tiles = (a->n + BN - 1) / BN;
  d.n_work = d.m_tiles * d.n_tiles * d.split;
  d.trace = g_trace_next ? 1 : 0;
  g_trace_next = 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (geglu) return launch_gemm_pair<BN, FVB_EPI_GEGLU>(ma, mb, mo, d, st);
  return launch_gemm_pair<BN, FVB_EPI_F32_ACC>(ma, mb, mo, d, st);
}


// Tensor-core attention for unsplit attention without suffix block masks
// (the SigLIP and Gemma prefix prefills); on unless FVB_ATTN_TC=0.
bool attn_tc_enabled() {
  static const int v = [] {
    const char* e = getenv("FVB_ATTN_TC");
    return e ? atoi(e) : 1;
  }();
  return v != 0;
}

template <int HD, int HDP, int NV>
int launch_attn_tc(const fvb_attn_args* a, const fvb::AttnDev& d,
                          cudaStream_t st) {
  namespace A = fvb::atc;
  using C = A::AtcCfg<HD, HDP, NV>;
  const long long kv_rows = (long long)(a->batch - 1) * a->kv_batch_rows + a->n_kv;
  // the maps span exactly the K / V heads' columns of each row, so a box
  // reaching past the last head reads zeros instead of memory beyond the view
  const int kv_heads = a->heads / a->group;
  const long long k_cols = (long long)(kv_heads - 1) * a->k_head_stride + a->head_dim;
  const long long v_cols = (long long)(kv_heads - 1) * a->v_head_stride + a->head_dim;
  CUtensorMap mk, mv;
  int r = make_map(&mk, a->k, kv_rows, k_cols, a->k_row_stride, A::BKV);
  if (!r) r = make_map(&mv, a->v, kv_rows, v_cols, a->v_row_stride, A::BKV);
  if (r) return r;
  A::AtcDev p;
  p.q = d.q; p.q_rs = d.q_rs; p.q_hs = d.q_hs;
  p.o = d.o; p.o_rs = d.o_rs; p.o_hs = d.o_hs;
  p.k_hs = (int)a->k_head_stride; p.v_hs = (int)a->v_head_stride;
  p.n_q = a->n_q; p.n_kv = a->n_kv; p.group = a->group;
  p.q_br = a->q_batch_rows; p.kv_br = a->kv_batch_rows;
  p.scale_log2 = d.scale_log2;
  p.key_valid = a->key_valid;
  p.heads = a->heads;
  p.splits = d.splits;
  p.blocks_per_split = d.blocks_per_split;
  p.part_o = d.part_o;
  p.part_ml = d.part_ml;
  p.trace = g_trace_next;
  g_trace_next = 0;
  auto kern = A::attn_tc_kernel<HD, HDP, NV>;
  if (int rr = ensure_smem(reinterpret_cast<const void*>(kern), C::SMEM, "attention")) return rr;
  const int tiles = (a->group * a->n_q + A::BM - 1) / A::BM;
  return launch_k("fvb_attention", kern,
                  dim3(tiles, a->heads / a->group, a->batch * d.splits),
                  dim3(A::THREADS), (size_t)C::SMEM, st, mk, mv, p);
}


bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

int fvb_version(void) { return 1; }
const char* fvb_last_error(void) { return g_err; }
int64_t fvb_launch_count(void) { return g_launches.load(); }

int fvb_get_device_status(int* status, int reset) {
  if (!status) return fail(FVB_ERR_INVALID_ARG, "status is NULL");
  cudaError_t e = cudaMemcpyFromSymbol(status, g_fvb_device_status, sizeof(int));
  if (e != cudaSuccess)
    return fail(FVB_ERR_CUDA, "read status: %s", cudaGetErrorString(e));
  if (reset) {
    int z = 0;
    e = cudaMemcpyToSymbol(g_fvb_device_status, &z, sizeof(int));
    if (e != cudaSuccess)
      return fail(FVB_ERR_CUDA, "reset status: %s", cudaGetErrorString(e));
  }
  return FVB_OK;
}

int fvb_probe_wait_timeout(int64_t limit_ns, int* gave_up_host, void* stream) {
  if (!gave_up_host) return fail(FVB_ERR_INVALID_ARG, "gave_up_host is NULL");
  if (limit_ns < 1000000) limit_ns = 1000000;
  if (limit_ns > (int64_t)FVB_WAIT_LIMIT_NS) limit_ns = (int64_t)FVB_WAIT_LIMIT_NS;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int* d = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&d), fvb::g_probe_result) != cudaSuccess)
    return fail(FVB_ERR_CUDA, "probe: symbol lookup failed");
  fvb::wait_timeout_probe_kernel<<<1, 32, 0, st>>>((unsigned long long)limit_ns, d);
  int r = check_launch("fvb_probe_wait_timeout");
  if (!r && cudaMemcpyAsync(gave_up_host, d, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    r = fail(FVB_ERR_CUDA, "probe: copy failed");
  if (!r && cudaStreamSynchronize(st) != cudaSuccess)
    r = fail(FVB_ERR_CUDA, "probe: %s", cudaGetErrorString(cudaGetLastError()));
  return r;
}

int fvb_gemm_trace_next(void) {
  g_trace_next = 1;
  return FVB_OK;
}

int fvb_expert_trace_read(uint64_t* host_out, int32_t max_ctas) {
  if (!host_out || max_ctas <= 0)
    return fail(FVB_ERR_INVALID_ARG, "fvb_expert_trace_read: bad arguments");
  const int n = max_ctas < 256 ? max_ctas : 256;
  cudaError_t e = cudaMemcpyFromSymbol(host_out, fvb::mega::g_mega_trace,
                                       (size_t)n * 32 * sizeof(uint64_t));
  if (e != cudaSuccess)
    return fail(FVB_ERR_CUDA, "trace read: %s", cudaGetErrorString(e));
  return FVB_OK;
}

int fvb_gemm_trace_read(uint64_t* host_out, int32_t max_ctas) {
  if (!host_out || max_ctas <= 0)
    return fail(FVB_ERR_INVALID_ARG, "fvb_gemm_trace_read: bad arguments");
  const int n = max_ctas < fvb::GEMM_TRACE_CTAS ? max_ctas : fvb::GEMM_TRACE_CTAS;
  cudaError_t e = cudaMemcpyFromSymbol(host_out, fvb::g_gemm_trace,
                                       (size_t)n * 16 * sizeof(uint64_t));
  if (e != cudaSuccess)
    return fail(FVB_ERR_CUDA, "trace read: %s", cudaGetErrorString(e));
  return FVB_OK;
}

int64_t fvb_gemm_workspace_bytes(const fvb_gemm_args* a) {
  if (!a || a->m <= 0 || a->n <= 0) return -1;
  if (!a->swap || a->epilogue == FVB_EPI_F32_ACC) return 0;
  const long long tiles = ((a->m + fvb::GEMM_BM - 1) / fvb::GEMM_BM) *
                          ((a->n + 63) / 64);
  return tiles * (64 * fvb::GEMM_BM * 4 + 4);
}

int fvb_gemm(const fvb_gemm_args* a, void* stream) {
  if (!a) return fail(FVB_ERR_INVALID_ARG, "args is NULL");
  if (!a->a || !a->b || !a->out)
    return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: NULL operand");
  if (a->m <= 0 || a->n <= 0 || a->k <= 0)
    return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: bad shape %d %d %d", a->m,
                a->n, a->k);
  if (a->k % 8 || a->lda % 8 || a->ldb % 8 || a->lda < a->k || a->ldb < a->k)
    return fail(FVB_ERR_INVALID_ARG,
                "fvb_gemm: k / lda / ldb must be multiples of 8 and >= k");
  if (!aligned16(a->a) || !aligned16(a->b))
    return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: operands must be 16B aligned");
  if (a->epilogue < FVB_EPI_BF16 || a->epilogue > FVB_EPI_QKV_ROPE)
    return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: bad epilogue %d", a->epilogue);
  const int n_feat = a->swap ? a->m : a->n;
  if (a->epilogue == FVB_EPI_GEGLU && (n_feat & 1))
    return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: GEGLU needs an even feature count");
  if (a->epilogue == FVB_EPI_QKV_ROPE) {
    if (!a->k_out || !a->v_out || !a->rope_cs || !a->positions ||
        a->head_dim % 16 || a->head_dim <= 0 ||
        n_feat != (a->n_heads + 2) * a->head_dim)
      return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: bad QKV_ROPE arguments");
    if (!a->swap && (a->ldo % 8 || a->ld_kv % 8 || !aligned16(a->out) ||
                     !aligned16(a->k_out) || !aligned16(a->v_out)))
      return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: QKV outputs must be 16B aligned");
  }
  if (a->epilogue == FVB_EPI_GEGLU && !a->swap &&
      (a->ldo % 8 || !aligned16(a->out)))
    return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: GEGLU output must be 16B aligned");
  if (a->row_add && a->row_add_mod <= 0)
    return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: row_add_mod must be > 0");
  if (a->res || a->gate_tok) {
    if (a->epilogue != FVB_EPI_BF16 || a->swap || a->pair || a->split_k > 1 ||
        a->n % 8 || (a->res && (a->ld_res % 8 || !aligned16(a->res))) ||
        (a->gate_tok && (a->ld_gate_tok % 8 || !aligned16(a->gate_tok))))
      return fail(FVB_ERR_INVALID_ARG,
                  "fvb_gemm: res / gate_tok need FVB_EPI_BF16, normal orientation, "
                  "one K split, n and row strides multiples of 8, 16B-aligned rows");
  }
  if (a->rope_interleaved && (a->epilogue != FVB_EPI_QKV_ROPE || a->swap))
    return fail(FVB_ERR_INVALID_ARG,
                "fvb_gemm: rope_interleaved needs FVB_EPI_QKV_ROPE, normal orientation");

  if (a->pair) return gemm_pair(a, stream);

  int bn = a->block_n;
  if (bn == 0) bn = a->swap ? 64 : 128;
  if (a->swap) {
    if (a->block_n != 0 && a->block_n != 64)
      return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: swap uses block_n 64");
    bn = 64;
  } else if (!aligned16(a->out) ||
             ((a->epilogue == FVB_EPI_QKV_ROPE) && (a->n % 32 || a->head_dim % 32))) {
    return fail(FVB_ERR_INVALID_ARG,
                "fvb_gemm: output must be 16B aligned (QKV: n, head_dim "
                "multiples of 32)");
  }
  if (bn != 64 && bn != 128 && bn != 192 && bn != 256)
    return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: block_n must be 64/128/192/256");

  // K splits: F32_ACC adds atomically into its output; a swapped GEMM with
  // any other epilogue reduces its splits in the workspace
  const int k_tiles = (a->k + fvb::GEMM_BK - 1) / fvb::GEMM_BK;
  const int tiles_mn = ((a->m + fvb::GEMM_BM - 1) / fvb::GEMM_BM) * ((a->n + bn - 1) / bn);
  const bool ws_split = a->swap && a->epilogue != FVB_EPI_F32_ACC;
  int split = a->split_k;
  if (split <= 0) {
    split = 1;
    if (a->swap && (!ws_split || a->workspace))
      split = sm_count() / tiles_mn > 1 ? sm_count() / tiles_mn : 1;
  }
  if (split > k_tiles) split = k_tiles;
  int kt_per_split = (k_tiles + split - 1) / split;
  split = (k_tiles + kt_per_split - 1) / kt_per_split;
  if (split > 1 && a->epilogue != FVB_EPI_F32_ACC) {
    if (!a->swap)
      return fail(FVB_ERR_INVALID_ARG,
                  "fvb_gemm: split_k > 1 needs FVB_EPI_F32_ACC or swap");
    const long long need = (long long)tiles_mn * (bn * fvb::GEMM_BM * 4 + 4);
    if (!a->workspace || a->workspace_bytes < need || !aligned16(a->workspace))
      return fail(FVB_ERR_WORKSPACE,
                  "fvb_gemm: split-K needs a zero-filled %lld-byte workspace", need);
  }

  CUtensorMap ma, mb;
  int r = make_map(&ma, a->a, a->m, a->k, a->lda, fvb::GEMM_BM);
  if (r) return r;
  r = make_map(&mb, a->b, a->n, a->k, a->ldb, bn);
  if (r) return r;

  fvb::GemmDev d;
  d.m = a->m; d.n = a->n; d.k = a->k;
  d.act = a->act;
  d.k_tiles = k_tiles;
  d.kt_per_split = kt_per_split;
  d.split = split;
  d.ws = reinterpret_cast<float*>(a->workspace);
  d.ws_cnt = d.ws ? reinterpret_cast<unsigned*>(
                        d.ws + (long long)tiles_mn * bn * fvb::GEMM_BM)
                  : nullptr;
  d.out = a->out; d.ldo = a->ldo;
  d.bias = a->bias; d.gate = a->gate; d.alpha = a->alpha;
  d.row_add = reinterpret_cast<const bf16*>(a->row_add);
  d.row_add_mod = a->row_add_mod;
  d.k_out = reinterpret_cast<bf16*>(a->k_out);
  d.v_out = reinterpret_cast<bf16*>(a->v_out);
  d.ld_kv = a->ld_kv; d.n_heads = a->n_heads; d.head_dim = a->head_dim;
  d.rope_cs = a->rope_cs; d.positions = a->positions;
  d.res = reinterpret_cast<const bf16*>(a->res); d.ld_res = a->ld_res;
  d.gate_tok = reinterpret_cast<const bf16*>(a->gate_tok); d.ld_gate_tok = a->ld_gate_tok;
  d.rope_interleaved = a->rope_interleaved;
  d.trace = g_trace_next ? 1 : 0;
  g_trace_next = 0;

  d.norm_out = reinterpret_cast<bf16*>(a->norm_out);
  d.ld_norm_out = a->ld_norm_out;
  d.norm_w = reinterpret_cast<const bf16*>(a->norm_w);
  d.norm_b = reinterpret_cast<const bf16*>(a->norm_b);
  d.norm_eps = a->norm_eps;
  d.norm_mode = a->norm_mode;
  d.norm_sync = reinterpret_cast<unsigned long long*>(a->norm_sync);
  if (a->norm_out) {
    const bool f32_out = a->epilogue == FVB_EPI_F32_ACC ||
                         (a->epilogue == FVB_EPI_F32_STORE && !a->row_add);
    if (a->swap || !f32_out || a->n % 128 || a->n > 2048 || a->ldo % 4 ||
        !a->norm_w || !a->norm_sync || (reinterpret_cast<uintptr_t>(a->norm_sync) & 7) ||
        (a->norm_mode != FVB_NORM_GEMMA_RMS && a->norm_mode != FVB_NORM_LAYER) ||
        (a->norm_mode == FVB_NORM_LAYER && !a->norm_b) || a->ld_norm_out % 4 ||
        (reinterpret_cast<uintptr_t>(a->norm_out) & 7) ||
        (reinterpret_cast<uintptr_t>(a->norm_w) & 7) ||
        (a->norm_b && (reinterpret_cast<uintptr_t>(a->norm_b) & 7)))
      return fail(FVB_ERR_INVALID_ARG, "fvb_gemm: unsupported fused norm arguments");
  }

  // TMA-store epilogue: normal orientation, plain row-major output rows on
  // 16-byte boundaries (the position-embedding add and QKV+RoPE keep the
  // per-row write-back)
  CUtensorMap mo;
  memset(&mo, 0, sizeof(mo));
  d.tma_out = 0;
  if (!a->swap && tma_out_enabled() && aligned16(a->out) && !a->res && !a->gate_tok) {
    const int e = a->epilogue;
    const bool f32 = e == FVB_EPI_F32_ACC || (e == FVB_EPI_F32_STORE && !a->row_add);
    const bool b16 = e == FVB_EPI_BF16 || e == FVB_EPI_GEGLU;
    if ((f32 && a->ldo % 4 == 0) || (b16 && a->ldo % 8 == 0)) {
      const int64_t cols = e == FVB_EPI_GEGLU ? a->n / 2 : a->n;
      const int box_cols = (f32 || e == FVB_EPI_GEGLU) ? 16 : 32;
      r = make_out_map(&mo, a->out, f32, a->m, cols, a->ldo, box_cols);
      if (r) return r;
      d.tma_out = 1;
    }
  }

  d.m_tiles = (a->m + fvb::GEMM_BM - 1) / fvb::GEMM_BM;
  d.n_tiles = (a->n + bn - 1) / bn;
  d.n_work = d.m_tiles * d.n_tiles * d.split;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define FVB_EPI_CASES(BN, SWAP)                                            \
  switch (a->epilogue) {                                                   \
    case FVB_EPI_BF16:                                                     \
      if (a->act == FVB_ACT_GELU_TANH)                                     \
        return launch_gemm<BN, FVB_EPI_BF16, SWAP, FVB_ACT_GELU_TANH>(ma, mb, mo, d, st); \
      if (a->act == FVB_ACT_SILU)                                          \
        return launch_gemm<BN, FVB_EPI_BF16, SWAP, FVB_ACT_SILU>(ma, mb, mo, d, st); \
      return launch_gemm<BN, FVB_EPI_BF16, SWAP>(ma, mb, mo, d, st);           \
    case FVB_EPI_F32_STORE: return launch_gemm<BN, FVB_EPI_F32_STORE, SWAP>(ma, mb, mo, d, st); \
    case FVB_EPI_F32_ACC: return launch_gemm<BN, FVB_EPI_F32_ACC, SWAP>(ma, mb, mo, d, st); \
    case FVB_EPI_GEGLU: return launch_gemm<BN, FVB_EPI_GEGLU, SWAP>(ma, mb, mo, d, st); \
    default: return launch_gemm<BN, FVB_EPI_QKV_ROPE, SWAP>(ma, mb, mo, d, st); \
  }
  if (a->swap) FVB_EPI_CASES(64, true)
  if (bn == 64) FVB_EPI_CASES(64, false)
  if (bn == 128) FVB_EPI_CASES(128, false)
  if (bn == 192) FVB_EPI_CASES(192, false)
  FVB_EPI_CASES(256, false)
#undef FVB_EPI_CASES
}

static int attn_prepare(const fvb_attn_args* a, fvb::AttnDev* d) {
  if (!a) return fail(FVB_ERR_INVALID_ARG, "args is NULL");
  if (!a->q || !a->k || !a->v || !a->o)
    return fail(FVB_ERR_INVALID_ARG, "fvb_attention: NULL operand");
  if (a->head_dim != 256 && a->head_dim != 72)
    return fail(FVB_ERR_UNSUPPORTED, "fvb_attention: head_dim %d (256 or 72)",
                a->head_dim);
  if (a->n_q <= 0 || a->n_kv <= 0 || a->heads <= 0 || a->group <= 0 ||
      a->heads % a->group || a->batch <= 0)
    return fail(FVB_ERR_INVALID_ARG, "fvb_attention: bad shape");
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) ||
      a->q_row_stride % 8 || a->k_row_stride % 8 || a->v_row_stride % 8 ||
      a->q_head_stride % 8 || a->k_head_stride % 8 || a->v_head_stride % 8)
    return fail(FVB_ERR_INVALID_ARG, "fvb_attention: 16B alignment required");
  if (a->o_row_stride % 2 || a->o_head_stride % 2)
    return fail(FVB_ERR_INVALID_ARG, "fvb_attention: output strides must be even");
  if (a->n_prefix < a->n_kv && a->q_block && !a->k_block)
    return fail(FVB_ERR_INVALID_ARG, "fvb_attention: q_block needs k_block");
  d->q = (const bf16*)a->q; d->q_rs = a->q_row_stride; d->q_hs = a->q_head_stride;
  d->k = (const bf16*)a->k; d->k_rs = a->k_row_stride; d->k_hs = a->k_head_stride;
  d->v = (const bf16*)a->v; d->v_rs = a->v_row_stride; d->v_hs = a->v_head_stride;
  d->o = (bf16*)a->o; d->o_rs = a->o_row_stride; d->o_hs = a->o_head_stride;
  d->n_q = a->n_q; d->n_kv = a->n_kv; d->heads = a->heads;
  d->group = a->group; d->batch = a->batch;
  d->q_br = a->q_batch_rows; d->kv_br = a->kv_batch_rows;
  d->scale_log2 = a->scale * 1.4426950408889634f;
  d->key_valid = a->key_valid; d->n_prefix = a->n_prefix;
  d->q_block = a->q_block; d->k_block = a->k_block;
  const int nkb = (a->n_kv + fvb::ATT_BN - 1) / fvb::ATT_BN;
  int splits = a->kv_splits > 1 ? a->kv_splits : 1;
  if (splits > nkb) splits = nkb;
  if (splits > fvb::ATT_MAX_SPLITS) splits = fvb::ATT_MAX_SPLITS;
  d->blocks_per_split = (nkb + splits - 1) / splits;
  d->splits = (nkb + d->blocks_per_split - 1) / d->blocks_per_split;
  const long long rows = (long long)a->batch * a->heads * a->n_q;
  d->part_o = (float*)a->workspace;
  d->part_ml = d->part_o ? d->part_o + (long long)d->splits * rows * a->head_dim
                         : nullptr;
  return FVB_OK;
}

int64_t fvb_attention_workspace_bytes(const fvb_attn_args* a) {
  fvb::AttnDev d;
  if (attn_prepare(a, &d)) return -1;
  if (d.splits == 1) return 0;
  const long long rows = (long long)a->batch * a->heads * a->n_q;
  return (long long)d.splits * rows * (a->head_dim + 2) * sizeof(float);
}

int fvb_attention(const fvb_attn_args* a, void* stream) {
  fvb::AttnDev d;
  int r = attn_prepare(a, &d);
  if (r) return r;
  if (d.splits > 1) {
    const long long need = fvb_attention_workspace_bytes(a);
    if (!a->workspace || a->workspace_bytes < need || !aligned16(a->workspace))
      return fail(FVB_ERR_WORKSPACE, "fvb_attention: workspace needs %lld bytes",
                  need);
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (a->n_prefix >= a->n_kv && a->n_kv <= fvb::atc::MAX_KEYS &&
      attn_tc_enabled() &&
      aligned16(a->o) && a->o_row_stride % 8 == 0 && a->o_head_stride % 8 == 0) {
    if (a->head_dim == 256) return launch_attn_tc<256, 256, 256>(a, d, st);
    return launch_attn_tc<72, 128, 80>(a, d, st);
  }
  dim3 grid((a->n_q + fvb::ATT_BM - 1) / fvb::ATT_BM, a->heads,
            a->batch * d.splits);
  if (a->head_dim == 256) {
    constexpr int S = fvb::attn_smem_bytes<256, 256>();
    if (int rr = ensure_smem(reinterpret_cast<const void*>(fvb::attn_kernel<256, 256>), S, "fvb_attention")) return rr;
    return launch_k("fvb_attention", fvb::attn_kernel<256, 256>, grid,
                    dim3(fvb::ATT_THREADS), (size_t)S, st, d);
  } else {
    constexpr int S = fvb::attn_smem_bytes<72, 80>();
    if (int rr = ensure_smem(reinterpret_cast<const void*>(fvb::attn_kernel<72, 80>), S, "fvb_attention")) return rr;
    return launch_k("fvb_attention", fvb::attn_kernel<72, 80>, grid,
                    dim3(fvb::ATT_THREADS), (size_t)S, st, d);
  }
}

int fvb_attention_combine(const fvb_attn_args* a, void* stream) {
  fvb::AttnDev d;
  int r = attn_prepare(a, &d);
  if (r) return r;
  if (d.splits == 1) return FVB_OK;
  if (!a->workspace) return fail(FVB_ERR_WORKSPACE, "combine: no workspace");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int rows = a->batch * a->heads * a->n_q;
  if (a->head_dim == 256)
    return launch_k("fvb_attention_combine", fvb::attn_combine_kernel<256>,
                    dim3(rows), dim3(256), 0, st, d);
  return launch_k("fvb_attention_combine", fvb::attn_combine_kernel<72>,
                  dim3(rows), dim3(96), 0, st, d);
}

int fvb_norm(int32_t mode, const float* x, int64_t ld_in, void* out,
             int64_t ld_out, int32_t out_f32, int32_t rows, int32_t dim,
             const void* w, const void* b, const float* mod, float eps,
             void* stream) {
  if (!x || !out || rows <= 0 || dim <= 0 || dim % 4 || ld_in % 4 ||
      ld_out % 4)
    return fail(FVB_ERR_INVALID_ARG, "fvb_norm: bad arguments");
  if (mode == FVB_NORM_GEMMA_RMS && !w)
    return fail(FVB_ERR_INVALID_ARG, "fvb_norm: weight required");
  if (mode == FVB_NORM_ADA_RMS && !mod)
    return fail(FVB_ERR_INVALID_ARG, "fvb_norm: modulation required");
  if (mode == FVB_NORM_LAYER && (!w || !b))
    return fail(FVB_ERR_INVALID_ARG, "fvb_norm: weight and bias required");
  if (mode < 0 || mode > 2)
    return fail(FVB_ERR_INVALID_ARG, "fvb_norm: bad mode");
  if (dim % 128 == 0 && dim <= 2048 && rows >= 64) {
    const dim3 grid((rows + fvb::NORM_ROWS_PER_CTA - 1) / fvb::NORM_ROWS_PER_CTA);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define FVB_NORM_WARP(V)                                                      \
  return launch_k("fvb_norm", fvb::norm_warp_kernel<V>, grid, dim3(256), 0,   \
                  st, (int)mode, x, (long long)ld_in, out, (long long)ld_out, \
                  (int)out_f32, (int)rows, (int)dim, (const bf16*)w,          \
                  (const bf16*)b, mod, eps);
    switch (dim / 128) {
      case 1: FVB_NORM_WARP(1)
      case 2: FVB_NORM_WARP(2)
      case 4: FVB_NORM_WARP(4)
      case 8: FVB_NORM_WARP(8)
      case 9: FVB_NORM_WARP(9)
      case 16: FVB_NORM_WARP(16)
      default: break;
    }
#undef FVB_NORM_WARP
  }
  return launch_k("fvb_norm", fvb::norm_kernel, dim3(rows),
                  dim3(fvb::NORM_THREADS), 0,
                  reinterpret_cast<cudaStream_t>(stream), (int)mode, x,
                  (long long)ld_in, out, (long long)ld_out, (int)out_f32,
                  (int)dim, (const bf16*)w, (const bf16*)b, mod, eps);
}

int fvb_norm_bf16(int32_t mode, const void* x, int64_t ld_in, void* out,
                  int64_t ld_out, int32_t rows, int32_t dim, const void* w,
                  const void* b, const void* style, void* gate_out,
                  int64_t ld_gate, float eps, void* stream) {
  if (!x || !out || rows <= 0 || dim <= 0 || dim % 8 || ld_in % 8 || ld_out % 8 ||
      !aligned16(x) || !aligned16(out))
    return fail(FVB_ERR_INVALID_ARG, "fvb_norm_bf16: bad arguments");
  if (mode == FVB_NORM_LAYER && (!w || !b || !aligned16(w) || !aligned16(b)))
    return fail(FVB_ERR_INVALID_ARG, "fvb_norm_bf16: weight and bias required");
  if (mode == FVB_NORM_ADA_STYLE &&
      (!style || !gate_out || !aligned16(style) || !aligned16(gate_out) || ld_gate % 8))
    return fail(FVB_ERR_INVALID_ARG, "fvb_norm_bf16: style and gate output required");
  if (mode != FVB_NORM_RMS && mode != FVB_NORM_LAYER && mode != FVB_NORM_ADA_STYLE)
    return fail(FVB_ERR_INVALID_ARG, "fvb_norm_bf16: bad mode");
  return launch_k("fvb_norm_bf16", fvb::norm_bf16_kernel, dim3((rows + 7) / 8), dim3(256),
                  0, reinterpret_cast<cudaStream_t>(stream), (int)mode, (const bf16*)x,
                  (long long)ld_in, (bf16*)out, (long long)ld_out, (int)rows, (int)dim,
                  (const bf16*)w, (const bf16*)b, (const bf16*)style, (bf16*)gate_out,
                  (long long)ld_gate, eps);
}

int fvb_softmax_rows(const float* logits, int64_t ld_in, int32_t rows,
                     int32_t keys, int32_t n_prefix, const int32_t* valid_prefix,
                     void* out, int64_t ld_out, void* stream) {
  if (!logits || !out || !valid_prefix || rows <= 0 || keys <= 0 || n_prefix < 0 ||
      n_prefix > keys || ld_in < keys || ld_out < keys)
    return fail(FVB_ERR_INVALID_ARG, "fvb_softmax_rows: bad arguments");
  return launch_k("fvb_softmax_rows", fvb::softmax_rows_kernel, dim3((rows + 7) / 8),
                  dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), logits,
                  (long long)ld_in, (int)rows, (int)keys, (int)n_prefix,
                  (const int*)valid_prefix, (bf16*)out, (long long)ld_out);
}

int fvb_patchify(const uint8_t* images, int32_t views, int32_t height,
                 int32_t width, int32_t patch, const float* mean3,
                 const float* std3, void* out, int64_t ldo, void* stream) {
  if (!images || !out || !mean3 || !std3 || views <= 0 || patch <= 0 ||
      height % patch || width % patch || ldo < 3 * patch * patch)
    return fail(FVB_ERR_INVALID_ARG, "fvb_patchify: bad arguments");
  const int rows = views * (height / patch) * (width / patch);
  return launch_k("fvb_patchify", fvb::patchify_kernel, dim3(rows), dim3(256),
                  0, reinterpret_cast<cudaStream_t>(stream), images,
                  (int)height, (int)width, (int)patch, mean3[0], mean3[1],
                  mean3[2], std3[0], std3[1], std3[2], (bf16*)out,
                  (long long)ldo);
}

int fvb_patchify_f32(const float* pixels, int32_t views, int32_t height,
                     int32_t width, int32_t patch, void* out, int64_t ldo,
                     void* stream) {
  if (!pixels || !out || views <= 0 || patch <= 0 || height % patch ||
      width % patch || ldo < 3 * patch * patch)
    return fail(FVB_ERR_INVALID_ARG, "fvb_patchify_f32: bad arguments");
  const int rows = views * (height / patch) * (width / patch);
  return launch_k("fvb_patchify_f32", fvb::patchify_f32_kernel, dim3(rows),
                  dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), pixels,
                  (int)height, (int)width, (int)patch, (bf16*)out,
                  (long long)ldo);
}

int fvb_resize_patchify(const uint8_t* images, int32_t views,
                        int32_t src_height, int32_t src_width, int32_t size,
                        int32_t patch, const float* mean3, const float* std3,
                        void* out, int64_t ldo, void* stream) {
  if (!images || !out || !mean3 || !std3 || views <= 0 || patch <= 0 ||
      size <= 0 || size % patch || src_height <= 0 || src_width <= 0 ||
      ldo < 3 * patch * patch)
    return fail(FVB_ERR_INVALID_ARG, "fvb_resize_patchify: bad arguments");
  const int rows = views * (size / patch) * (size / patch);
  return launch_k("fvb_resize_patchify", fvb::resize_patchify_kernel, dim3(rows),
                  dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), images,
                  (int)src_height, (int)src_width, (int)size, (int)patch, mean3[0],
                  mean3[1], mean3[2], std3[0], std3[1], std3[2], (bf16*)out,
                  (long long)ldo);
}

int fvb_embed_tokens(const int64_t* ids, int32_t n, const void* table,
                     int32_t dim, float scale, float* out, int64_t ldo,
                     void* stream) {
  if (!ids || !table || !out || n <= 0 || dim <= 0)
    return fail(FVB_ERR_INVALID_ARG, "fvb_embed_tokens: bad arguments");
  return launch_k("fvb_embed_tokens", fvb::embed_kernel, dim3(n), dim3(256),
                  0, reinterpret_cast<cudaStream_t>(stream),
                  (const long long*)ids, (const bf16*)table, (int)dim, scale,
                  out, (long long)ldo);
}

int fvb_small_linear(const float* x, int64_t ldx, int32_t t, int32_t k,
                     const void* w, int64_t ldw, int32_t n, const float* bias,
                     int32_t act, int32_t mode, float alpha, void* out,
                     int64_t ldo, void* stream) {
  if (!x || !w || !out || t <= 0 || k <= 0 || n <= 0 || mode < 0 || mode > 2)
    return fail(FVB_ERR_INVALID_ARG, "fvb_small_linear: bad arguments");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = aligned16(w) && ldw % 8 == 0;
  if (vec && k % 8 == 0 && k <= 64)
    return launch_k("fvb_small_linear", fvb::small_linear_narrow_kernel,
                    dim3((unsigned)((long long)t * ((n + 255) / 256))), dim3(256), 0, st,
                    x, (long long)ldx, (int)k, (const bf16*)w, (long long)ldw,
                    (int)n, bias, (int)act, (int)mode, alpha, out, (long long)ldo);
  if (vec && k % 256 == 0 && aligned16(x) && ldx % 4 == 0)
    return launch_k("fvb_small_linear", fvb::small_linear_wide_kernel,
                    dim3((unsigned)(((long long)t * n * 32 + 255) / 256)), dim3(256), 0,
                    st, x, (long long)ldx, (int)t, (int)k, (const bf16*)w,
                    (long long)ldw, (int)n, bias, (int)act, (int)mode, alpha, out,
                    (long long)ldo);
  const long long warps = (long long)t * n;
  const int threads = 256;
  const long long blocks = (warps * 32 + threads - 1) / threads;
  return launch_k("fvb_small_linear", fvb::small_linear_kernel,
                  dim3((unsigned)blocks), dim3(threads), 0,
                  reinterpret_cast<cudaStream_t>(stream), x, (long long)ldx,
                  (int)t, (int)k, (const bf16*)w, (long long)ldw, (int)n, bias,
                  (int)act, (int)mode, alpha, out, (long long)ldo);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Persistent expert step
// ---------------------------------------------------------------------------
namespace {

struct ExpertLayout {
  fvb::mega::Params p;
  long long bytes;
};

int expert_prepare(const fvb_expert_args* a, ExpertLayout* out) {
  using namespace fvb::mega;
  if (!a) return fail(FVB_ERR_INVALID_ARG, "args is NULL");
  if (a->n_layers <= 0 || a->n_layers > 64 || a->n_tok <= 0 || a->n_tok > TOK ||
      a->width % 128 || a->width <= 0 || a->mlp % 64 || a->mlp <= 0 ||
      a->head_dim != 256 || a->heads <= 0 || a->n_prefix < 0 ||
      (a->n_prefix + a->n_tok + 63) / 64 > MAX_NKB ||
      a->cache_rows < a->n_prefix + a->n_tok)
    return fail(FVB_ERR_INVALID_ARG, "fvb_expert_step: unsupported shape");
  Params& p = out->p;
  p.n_layers = a->n_layers; p.n_tok = a->n_tok; p.width = a->width;
  p.mlp = a->mlp; p.heads = a->heads; p.hd = a->head_dim;
  p.n_prefix = a->n_prefix;
  const int G = sm_count();
  const int rows[N_GEMM] = {(a->heads + 2) * a->head_dim, a->width, 2 * a->mlp,
                            a->width};
  const int ks[N_GEMM] = {a->width, a->heads * a->head_dim, a->width, a->mlp};
  for (int i = 0; i < N_GEMM; ++i) {
    Gemm& g = p.g[i];
    g.rows = rows[i];
    g.m_tiles = rows[i] / 128;
    g.k_tiles = ks[i] / 64;
    int sp = G / g.m_tiles > 1 ? G / g.m_tiles : 1;
    if (sp > g.k_tiles) sp = g.k_tiles;
    g.kt_per = (g.k_tiles + sp - 1) / sp;
    if (g.kt_per > MAX_KT) g.kt_per = MAX_KT;
    g.splits = (g.k_tiles + g.kt_per - 1) / g.kt_per;
    g.items = g.m_tiles * g.splits;
  }
  p.in_scale = a->in_scale; p.post_scale = a->post_scale;
  p.qkv_bias = a->qkv_bias; p.gu_bias = a->gu_bias;
  p.o_gate = a->o_gate; p.down_gate = a->down_gate;
  p.eps = a->eps; p.x = a->x;
  p.kc = (bf16*)a->k_cache; p.vc = (bf16*)a->v_cache;
  p.cache_layer = a->cache_rows * a->head_dim;
  p.key_valid = a->key_valid; p.blocks = a->blocks; p.positions = a->positions;
  p.rope_cs = a->rope_cs;
  p.rope_suf = a->rope_suffix;
  p.scale_log2 = (1.f / sqrtf((float)a->head_dim)) * 1.4426950408889634f;
  p.nkb = (a->n_prefix + a->n_tok + 63) / 64;
  p.trace = getenv("FVB_EXPERT_TRACE") ? 1 : 0;
  p.stages = STAGES;
  if (getenv("FVB_EXPERT_STAGES")) {
    const int v = atoi(getenv("FVB_EXPERT_STAGES"));
    if (v >= 1 && v <= STAGES) p.stages = v;
  }
  // workspace carve-up (256-byte aligned pieces)
  char* base = (char*)a->workspace;
  long long off = 0;
  auto take = [&](long long n) {
    long long o = off;
    off += (n + 255) & ~255ll;
    return base ? base + o : nullptr;
  };
  p.acc_qkv = (float*)take((long long)TOK * rows[0] * 4);
  p.acc_gu = (float*)take((long long)TOK * rows[2] * 4);
  p.ss_in = (float*)take(TOK * 4);
  p.ss_post = (float*)take(TOK * 4);
  p.part_o = (float*)take((long long)a->heads * p.nkb * TOK * a->head_dim * 4);
  p.part_ml = (float*)take((long long)a->heads * p.nkb * TOK * 2 * 4);
  p.attn = (bf16*)take((long long)TOK * a->heads * a->head_dim * 2);
  p.qb = (bf16*)take((long long)TOK * a->heads * a->head_dim * 2);
  p.xs = (bf16*)take((long long)TOK * a->width * 2);
  p.hb = (bf16*)take((long long)TOK * a->mlp * 2);
  p.bar = (unsigned*)take(BAR_WORDS * 4);
  out->bytes = off;
  return FVB_OK;
}

}  // namespace

extern "C" int64_t fvb_expert_workspace_bytes(const fvb_expert_args* a) {
  ExpertLayout L;
  fvb_expert_args tmp = *a;
  tmp.workspace = nullptr;
  if (expert_prepare(&tmp, &L)) return -1;
  return L.bytes;
}

extern "C" int fvb_expert_step(const fvb_expert_args* a, void* stream) {
  using namespace fvb::mega;
  ExpertLayout L;
  int r = expert_prepare(a, &L);
  if (r) return r;
  if (!a->w_qkv || !a->w_o || !a->w_gu || !a->w_down || !a->in_scale ||
      !a->post_scale || !a->x || !a->k_cache || !a->v_cache || !a->blocks ||
      !a->positions || !a->rope_cs || !a->rope_suffix)
    return fail(FVB_ERR_INVALID_ARG, "fvb_expert_step: NULL operand");
  if (!a->workspace || a->workspace_bytes < L.bytes || !aligned16(a->workspace))
    return fail(FVB_ERR_WORKSPACE, "fvb_expert_step: workspace needs %lld bytes",
                L.bytes);
  const Params& p = L.p;
  CUtensorMap maps[N_GEMM];
  const void* w[N_GEMM] = {a->w_qkv, a->w_o, a->w_gu, a->w_down};
  for (int i = 0; i < N_GEMM; ++i) {
    r = make_map(&maps[i], w[i], (long long)p.g[i].rows * a->n_layers,
                 (long long)p.g[i].k_tiles * 64, (long long)p.g[i].k_tiles * 64, 128);
    if (r) return r;
  }
  CUtensorMap bmaps[3];
  r = make_map(&bmaps[0], p.xs, TOK, a->width, a->width, TOK);
  if (!r) r = make_map(&bmaps[1], p.attn, TOK, (long long)a->heads * a->head_dim,
                       (long long)a->heads * a->head_dim, TOK);
  if (!r) r = make_map(&bmaps[2], p.hb, TOK, a->mlp, a->mlp, TOK);
  if (r) return r;
  // attention operands: head columns of the rotated queries, and 64-row
  // blocks of one layer's cache (3-D so that rows past the cache read zeros)
  CUtensorMap amaps[3];
  r = make_map(&amaps[0], p.qb, TOK, (long long)a->heads * a->head_dim,
               (long long)a->heads * a->head_dim, 64);
  if (!r) r = make_cache_map(&amaps[1], a->k_cache, a->n_layers, a->cache_rows, a->head_dim);
  if (!r) r = make_cache_map(&amaps[2], a->v_cache, a->n_layers, a->cache_rows, a->head_dim);
  if (r) return r;
  if (int rr = ensure_smem(reinterpret_cast<const void*>(expert_step_kernel), SMEM_BYTES, "expert")) return rr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count());
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeCooperative;
  attrs[0].val.cooperative = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  // the weight stream of the step starts under the previous kernel's tail
  // when the driver accepts a cooperative launch with programmatic
  // serialisation; otherwise the plain cooperative launch
  static int coop_pdl = -1;
  if (coop_pdl < 0) coop_pdl = pdl_enabled() ? 1 : 0;
  cfg.numAttrs = coop_pdl ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, expert_step_kernel, maps[0], maps[1],
                                     maps[2], maps[3], bmaps[0], bmaps[1],
                                     bmaps[2], amaps[0], amaps[1], amaps[2], p);
  if (e != cudaSuccess && coop_pdl) {
    cudaGetLastError();
    coop_pdl = 0;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, expert_step_kernel, maps[0], maps[1], maps[2], maps[3],
                           bmaps[0], bmaps[1], bmaps[2], amaps[0], amaps[1], amaps[2], p);
  }
  if (e != cudaSuccess)
    return fail(FVB_ERR_CUDA, "fvb_expert_step: launch failed: %s",
                cudaGetErrorString(e));
  return check_launch("fvb_expert_step");
}

// ---------------------------------------------------------------------------
// Allocation-free attention.
//
// Some callers cannot allocate device memory at all: an embedded robot
// controller whose memory budget is fixed at start-up, a process running
// under an allocator that forbids cudaMalloc after initialisation, or a
// foreign-language binding that has no way to hand us a device buffer.
// fvb_attention_noalloc serves them: the split-over-keys partial results
// live in the file-scope array below instead of a caller workspace.  Every
// GPU that loads this library reserves FVB_NOALLOC_SCRATCH_BYTES for it until
// the process exits.  All calls on a device share the one array; it keeps
// the last call's contents.  Nothing in it has to start at zero: every split
// writes all of its partial rows (empty key ranges write m = -inf, l = 0)
// before the combine reads them.  Calls whose kernels overlap on the GPU
// (different streams, or concurrent host threads) race on the array.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char
    g_noalloc_scratch[FVB_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch for the current device.  In host code
// the symbol name is only a host-side stand-in, so the address is looked up
// with cudaGetSymbolAddress (with that device current) on the first call on
// each device and cached together with the CUDA context it belongs to.  A
// cudaDeviceReset destroys that context and reloads the module, so a call
// that finds a different current context looks the address up again instead
// of reusing a stale pointer.  The first call on a device should come before
// any stream capture.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

static CUcontext current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  CUcontext c = nullptr;
  if (fn) fn(&c);
  return c;
}

static int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* ptrs[128] = {};
  static CUcontext ctxs[128] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(FVB_ERR_CUDA, "fvb_attention_noalloc: cudaGetDevice: %s",
                cudaGetErrorString(e));
  if (dev < 0 || dev >= 128)
    return fail(FVB_ERR_UNSUPPORTED, "fvb_attention_noalloc: device %d", dev);
  // a runtime call on the device binds its primary context before the
  // context handle is read
  int n_sm = 0;
  e = cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess)
    return fail(FVB_ERR_CUDA, "fvb_attention_noalloc: %s", cudaGetErrorString(e));
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev] || ctxs[dev] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(FVB_ERR_CUDA,
                  "fvb_attention_noalloc: cudaGetSymbolAddress: %s",
                  cudaGetErrorString(e));
    ptrs[dev] = p;
    ctxs[dev] = ctx;
  }
  *out = ptrs[dev];
  return FVB_OK;
}

extern "C" int fvb_attention_noalloc(const fvb_attn_args* a, void* stream) {
  fvb::AttnDev d;
  int r = attn_prepare(a, &d);
  if (r) return r;
  const long long rows = (long long)a->batch * a->heads * a->n_q;
  const long long need =
      d.splits > 1 ? (long long)d.splits * rows * (a->head_dim + 2) * 4 : 0;
  if (need > (long long)FVB_NOALLOC_SCRATCH_BYTES)
    return fail(FVB_ERR_WORKSPACE,
                "fvb_attention_noalloc: %d key splits x %lld query rows need "
                "%lld bytes of scratch, more than the %lld-byte limit; use "
                "fewer kv_splits or fvb_attention with a caller workspace",
                d.splits, rows, need, (long long)FVB_NOALLOC_SCRATCH_BYTES);
  void* ws = nullptr;
  if (d.splits > 1) {
    r = noalloc_scratch(&ws);
    if (r) return r;
  }
  d.part_o = (float*)ws;
  d.part_ml = ws ? d.part_o + (long long)d.splits * rows * a->head_dim
                 : nullptr;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid((a->n_q + fvb::ATT_BM - 1) / fvb::ATT_BM, a->heads,
            a->batch * d.splits);
  if (a->head_dim == 256) {
    constexpr int S = fvb::attn_smem_bytes<256, 256>();
    r = ensure_smem(reinterpret_cast<const void*>(fvb::attn_kernel<256, 256>), S,
                    "fvb_attention_noalloc");
    if (r) return r;
    fvb::attn_kernel<256, 256><<<grid, fvb::ATT_THREADS, S, st>>>(d);
  } else {
    constexpr int S = fvb::attn_smem_bytes<72, 80>();
    r = ensure_smem(reinterpret_cast<const void*>(fvb::attn_kernel<72, 80>), S,
                    "fvb_attention_noalloc");
    if (r) return r;
    fvb::attn_kernel<72, 80><<<grid, fvb::ATT_THREADS, S, st>>>(d);
  }
  r = check_launch("fvb_attention_noalloc");
  if (r || d.splits == 1) return r;
  if (a->head_dim == 256)
    fvb::attn_combine_kernel<256><<<(unsigned)rows, 256, 0, st>>>(d);
  else
    fvb::attn_combine_kernel<72><<<(unsigned)rows, 96, 0, st>>>(d);
  return check_launch("fvb_attention_noalloc (combine)");
}
