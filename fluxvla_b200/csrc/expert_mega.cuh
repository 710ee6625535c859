// Persistent expert-layer kernel for the denoise loop: all layers of one
// flow-matching step (action-expert Gemma stack over <= 64 suffix tokens) in
// one cooperative launch, one CTA per SM.
//
// Per layer, ten phases separated by grid barriers:
//   0 prep    xs[t,k] = bf16(x[t,k](1+w_in[k])), ss_in[t] += sum_k x^2
//   1 QKV     acc_qkv[t,f] += W_qkv[f,k] xs[t,k]  (split-K, f32 reductions;
//             B operand = xs by TMA)
//   2 finalize q,k,v = rope(rstd_in[t]*acc + bias) as bf16: q to qb, the
//             suffix k / v into the layer's cache rows n_prefix..
//   3 ATT     per (head, 64-key block): Q, K, V tiles by TMA, masked
//             attention over prefix + suffix keys -> bf16 partial, (max, sum)
//   4 merge   key-block partials -> attn[t, h*hd + d] (bf16)
//   5 O       x[t,f] += gate_o[f] * (W_o attn)  (split-K reductions)
//   6 prep    xs = bf16(x(1+w_post)), ss_post
//   7 GU      acc_gu[t,f] += W_gu[f,k] xs[t,k]
//   8 GeGLU   hb[t,i] = bf16(gelu(rs*g + bg) * (rs*u + bu)), rs = rstd_post
//   9 DOWN    x[t,f] += gate_d[f] * (W_down hb)
// Each phase costs about one L2 round trip plus one grid barrier; folding a
// reshaping phase into its consumer was measured slower (every consumer CTA
// then re-reads the f32 activations of its K slice).
// RMSNorm is linear in the un-normalised row apart from the per-token factor
// rstd, so the GEMM runs on x*(1+w) and rstd is applied by the consumer; for
// adaRMSNorm the shift enters as W*shift, precomputed per step (bias arrays).
//
// Roles: warp 0 lane 0 streams every weight tile of the step through a
// STAGES-deep TMA ring in a fixed order and never waits for a barrier (the
// weights do not depend on the previous phase); warp 1 lane 0 issues
// tcgen05.mma (M=128 weight rows, N=64 tokens, K=16) into a 64-column TMEM
// accumulator; warps 2..5 issue the B operand TMA (tokens x K-slice, bf16,
// 128-byte swizzle), run the epilogue reductions, the prep / finalize /
// merge phases and the attention, and take part in the grid barriers.
#pragma once

#include "attention.cuh"
#include "common.cuh"

namespace fvb {
namespace mega {

constexpr int THREADS = 192;
constexpr int STAGES = 6;
constexpr int TOK = 64;                    // MMA N (tokens, padded)
constexpr int A_BYTES = 128 * 64 * 2;      // weight k-tile (16 KB)
constexpr int BKT_BYTES = TOK * 64 * 2;    // B k-tile (8 KB)
constexpr int MAX_KT = 8;                  // k-tiles per work item
// attention tiles: 64 rows x 256 dims bf16 as four 64-column TMA boxes,
// 128-byte swizzled (8 KB each), Q | K | V back to back
constexpr int ATT_TILE_BYTES = 64 * 256 * 2;
constexpr int REGION_BYTES = 3 * ATT_TILE_BYTES + 64 + 64 * 4 + 2 * 64 * 4;  // >= MAX_KT*BKT
constexpr int SMEM_BYTES = 1024 + STAGES * A_BYTES + REGION_BYTES + 256 + TOK * 4;
constexpr int N_GEMM = 4;  // QKV, O, GU, DOWN

struct Gemm {
  int rows;        // weight rows per layer
  int k_tiles;     // K / 64
  int m_tiles;     // rows / 128
  int kt_per;      // k-tiles per item
  int splits;
  int items;       // m_tiles * splits
};

struct Params {
  int n_layers, n_tok, width, mlp, heads, hd, n_prefix;
  Gemm g[N_GEMM];
  const float* in_scale;    // [L, width]
  const float* post_scale;  // [L, width]
  const float* qkv_bias;    // [L, (H+2)*hd] or null
  const float* gu_bias;     // [L, 2*mlp] or null
  const float* o_gate;      // [L, width] or null
  const float* down_gate;   // [L, width] or null
  float eps;
  float* x;                 // residual [n_tok, width] f32
  bf16* kc;                 // [L, cache_rows, hd]: prefix rows read, the
  bf16* vc;                 // suffix rows n_prefix.. written each step
  long long cache_layer;    // elements per layer of the cache
  const uint8_t* key_valid;
  const int* blocks;
  const int* positions;
  const float* rope_cs;
  const float* rope_suf;    // [n_tok, hd/2, 2] cos/sin at the suffix positions
  float scale_log2;
  // workspace
  float* acc_qkv;  // [TOK, (H+2)*hd]
  float* acc_gu;   // [TOK, 2*mlp]
  float* ss_in;    // [TOK]
  float* ss_post;  // [TOK]
  float* part_o;   // [heads*nkb, TOK, hd] bf16, normalised per block
  float* part_ml;  // [heads*nkb, TOK, 2]
  bf16* attn;      // [TOK, heads*hd]
  bf16* qb;        // [TOK, heads*hd] rotated queries (rows >= n_tok zero)
  bf16* xs;        // [TOK, width] x*(1+w) for the QKV / gate-up B operand
  bf16* hb;        // [TOK, mlp] gelu(g)*u for the down B operand
  unsigned* bar;   // [0..1] 64-bit arrival count, [BAR_ABORT] abort flag
  int nkb;         // key blocks of 64
  int trace;       // diagnostics: phase stamps of layer 0 in g_mega_trace
  int stages;      // weight ring depth in use (<= STAGES)
};

// Diagnostics: per CTA, globaltimer at worker start, then after the work
// and after the barrier of each of the 10 phases of layer 0 (slots 24.. hold stamps inside the attention phase).
__device__ unsigned long long g_mega_trace[256][32];

// ---------------------------------------------------------------------------
// waits with a time limit and a shared abort flag
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool aborted(const Params& p) {
  return *reinterpret_cast<volatile unsigned*>(p.bar + 288) != 0u;
}

__device__ __forceinline__ void set_abort(const Params& p) {
  record_device_error(FVB_ERR_DEVICE_TIMEOUT);
  atomicExch(p.bar + 288, 1u);
}

__device__ __forceinline__ bool wait_bar(const Params& p, uint64_t* bar,
                                         uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 8; ++i)
      if (mbar_try_wait_sleep(addr, parity, 20000)) return true;
    if (aborted(p)) return false;
    if (globaltimer_ns() - t0 > FVB_WAIT_LIMIT_NS) {
      set_abort(p);
      return false;
    }
  }
}

__device__ __forceinline__ void bar128() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Grid barrier among the 4 worker warps of every CTA: one acquire-release
// 64-bit arrival counter (bar[0..1]) that only grows, polled with acquire
// loads: the k-th barrier of the workspace's history completes when it
// reaches (k+1)*gridDim.x, and each arrival learns k from the value it
// replaced (64 bits: no wrap-around in any realistic lifetime).  The abort
// flag bar[BAR_ABORT] is on its own line.
constexpr int BAR_ABORT = 288, BAR_WORDS = 320;
__device__ __forceinline__ unsigned long long ld_acquire64(const unsigned* a) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long atom_add_acq_rel64(unsigned* a) {
  unsigned long long old;
  asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], 1;"
               : "=l"(old) : "l"(a) : "memory");
  return old;
}
__device__ __forceinline__ void grid_sync(const Params& p, int wtid) {
  bar128();
  if (wtid == 0) {
    const unsigned long long G = gridDim.x;
    const unsigned long long old = atom_add_acq_rel64(p.bar);
    const unsigned long long target = (old / G + 1) * G;
    uint64_t t0 = 0;
    for (unsigned n = 0; ld_acquire64(p.bar) < target; ++n) {
      if ((n & 255) == 255) {
        if (aborted(p)) break;
        const uint64_t now = globaltimer_ns();
        if (t0 == 0) t0 = now;
        else if (now - t0 > FVB_WAIT_LIMIT_NS) { set_abort(p); break; }
      }
    }
  }
  bar128();
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ float4 ldcg4(const float* p) {
  return __ldcg(reinterpret_cast<const float4*>(p));
}

// byte offset of the 16-byte chunk (token t, k-chunk kc of 8) in the B
// operand (k-tile kc/8, 128-byte rows, 128-byte swizzle)
__device__ __forceinline__ int b_off(int t, int kc) {
  return (kc >> 3) * BKT_BYTES + t * 128 + (((kc & 7) ^ (t & 7)) << 4);
}

// ---------------------------------------------------------------------------
// attention block: 64 query rows (one head) x one 64-key block
// ---------------------------------------------------------------------------
// byte offset of element (row, col) of a 64 x 256 attention tile stored as
// four 64-column, 128-byte-swizzled TMA boxes (col a multiple of 8)
__device__ __forceinline__ uint32_t att_off(int row, int col) {
  return (uint32_t)((col >> 6) * 8192 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4));
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map,
                                            int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z),
      "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// attention block: 64 query rows (one head) x one 64-key block.  Operands by
// TMA: the rotated queries of head h (qb), and 64 keys / values from the
// layer's cache rows (prefix rows from the prefill, suffix rows written by
// the finalize phase; rows past the cache are zero-filled), completing on
// a_full (phase a_par).
// ---------------------------------------------------------------------------
__device__ void attention_item(const Params& p, int layer, int item,
                               uint8_t* region, uint64_t* a_full, uint32_t a_par,
                               const CUtensorMap* tm_q, const CUtensorMap* tm_k,
                               const CUtensorMap* tm_v, int wtid, bool tr) {
  const int hd = p.hd;
  const int h = item / p.nkb, kb = item % p.nkb;
  const int S = p.n_tok, E = p.n_prefix, n_kv = E + S;
  uint8_t* sQ = region;
  uint8_t* sK = region + ATT_TILE_BYTES;
  uint8_t* sV = region + 2 * ATT_TILE_BYTES;
  uint8_t* sMask = region + 3 * ATT_TILE_BYTES;
  int* sKb = reinterpret_cast<int*>(sMask + 64);

  const int key0 = kb * 64;
  if (wtid == 0) {
    mbar_arrive_expect_tx(a_full, 3 * ATT_TILE_BYTES);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      tma_load_2d(sQ + c * 8192, tm_q, h * hd + c * 64, 0, a_full);
      tma_load_3d(sK + c * 8192, tm_k, c * 64, key0, layer, a_full);
      tma_load_3d(sV + c * 8192, tm_v, c * 64, key0, layer, a_full);
    }
  }
  __syncwarp();
  if (wtid < 64) {
    const int key = key0 + wtid;
    uint8_t vis = key < n_kv;
    int kbv = 0;
    if (vis) {
      if (key < E) vis = p.key_valid ? (p.key_valid[key] != 0) : 1;
      else kbv = p.blocks[key - E];
    }
    sMask[wtid] = vis;
    sKb[wtid] = kbv;
  }
  // a wait that gives up has set the abort flag: the step's output is then
  // discarded, so the block is still computed (uniform control flow)
  wait_bar(p, a_full, a_par);
  bar128();
  if (tr) g_mega_trace[blockIdx.x][24] = globaltimer_ns();

  // S = Q K^T, masked online softmax over this block, O = P V
  const int warp = wtid >> 5, lane = wtid & 31;
  const int r0 = warp * 16 + (lane >> 2), r1 = r0 + 8;
  const int qb0 = r0 < S ? p.blocks[r0] : 0x7fffffff;
  const int qb1 = r1 < S ? p.blocks[r1] : 0x7fffffff;
  const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV);
  float s[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll 4
  for (int kk = 0; kk < 256 / 16; ++kk) {
    uint32_t a0, a1, a2, a3;
    ldsm_x4(sQa + att_off(warp * 16 + (lane & 15), kk * 16 + (lane >> 4) * 8),
            a0, a1, a2, a3);
#pragma unroll
    for (int nt = 0; nt < 8; nt += 2) {
      uint32_t b0, b1, b2, b3;
      const int mi = lane >> 3, rr = lane & 7;
      const int key = nt * 8 + (mi >> 1) * 8 + rr;
      ldsm_x4(sKa + att_off(key, kk * 16 + (mi & 1) * 8), b0, b1, b2, b3);
      mma_bf16_16816(s[nt], a0, a1, a2, a3, b0, b1);
      mma_bf16_16816(s[nt + 1], a0, a1, a2, a3, b2, b3);
    }
  }
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int kj = nt * 8 + (lane & 3) * 2 + e;
      const bool vis = sMask[kj] != 0;
      const bool pre = key0 + kj < E;
      const int kbv = sKb[kj];
      const bool v0 = vis && (pre || kbv <= qb0);
      const bool v1 = vis && (pre || kbv <= qb1);
      s[nt][e] = v0 ? s[nt][e] * p.scale_log2 : -INFINITY;
      s[nt][2 + e] = v1 ? s[nt][2 + e] * p.scale_log2 : -INFINITY;
      mx0 = fmaxf(mx0, s[nt][e]);
      mx1 = fmaxf(mx1, s[nt][2 + e]);
    }
  }
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
  }
  const float base0 = mx0 == -INFINITY ? 0.f : mx0;
  const float base1 = mx1 == -INFINITY ? 0.f : mx1;
  float l0 = 0.f, l1 = 0.f;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    s[nt][0] = exp2f(s[nt][0] - base0);
    s[nt][1] = exp2f(s[nt][1] - base0);
    s[nt][2] = exp2f(s[nt][2] - base1);
    s[nt][3] = exp2f(s[nt][3] - base1);
    l0 += s[nt][0] + s[nt][1];
    l1 += s[nt][2] + s[nt][3];
  }
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  if (tr) g_mega_trace[blockIdx.x][25] = globaltimer_ns();
  // partial output normalised by this block's row sum, as bf16 (the merge
  // weights it back by the sum): half the bytes of an f32 partial
  bf16* po = reinterpret_cast<bf16*>(p.part_o) + (long long)item * TOK * hd;
  float* pml = p.part_ml + (long long)item * TOK * 2;
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  // P V in four 64-column passes to bound registers
#pragma unroll 1
  for (int dp = 0; dp < 4; ++dp) {
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a0 = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        uint32_t b0, b1, b2, b3;
        const int mi = lane >> 3, rr = lane & 7;
        const int key = kk * 16 + (mi & 1) * 8 + rr;
        const int col = dp * 64 + nt * 8 + (mi >> 1) * 8;
        ldsm_x4_t(sVa + att_off(key, col), b0, b1, b2, b3);
        mma_bf16_16816(o[nt], a0, a1, a2, a3, b0, b1);
        mma_bf16_16816(o[nt + 1], a0, a1, a2, a3, b2, b3);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int d = dp * 64 + nt * 8 + (lane & 3) * 2;
      if (r0 < S)
        __stcg(reinterpret_cast<unsigned*>(po + (long long)r0 * hd + d),
               pack_bf16x2(o[nt][0] * inv0, o[nt][1] * inv0));
      if (r1 < S)
        __stcg(reinterpret_cast<unsigned*>(po + (long long)r1 * hd + d),
               pack_bf16x2(o[nt][2] * inv1, o[nt][3] * inv1));
    }
  }
  if ((lane & 3) == 0) {
    if (r0 < S) __stcg(reinterpret_cast<float2*>(pml + r0 * 2), make_float2(mx0, l0));
    if (r1 < S) __stcg(reinterpret_cast<float2*>(pml + r1 * 2), make_float2(mx1, l1));
  }
  if (tr) g_mega_trace[blockIdx.x][26] = globaltimer_ns();
  // the region is reused by the next item's TMA loads (async proxy)
  fence_async_smem();
  bar128();
}

// xs[t,k] = bf16(x[t,k]*scale[k]) and ss[t] += sum_k x[t,k]^2, spread over
// the grid (8 values per thread; a warp covers 256 values of one token)
__device__ void prep_scaled(const Params& p, const float* scale, float* ss,
                            int wtid) {
  const int per_tok = p.width / 8;
  const int total = p.n_tok * per_tok;
  const int lane = wtid & 31;
  for (int c = blockIdx.x * 128 + wtid; c - lane < total; c += gridDim.x * 128) {
    float q = 0.f;
    int t = 0;
    if (c < total) {
      t = c / per_tok;
      const int k = (c % per_tok) * 8;
      const float4 a = ldcg4(p.x + (long long)t * p.width + k);
      const float4 b = ldcg4(p.x + (long long)t * p.width + k + 4);
      const float4 sa = __ldg(reinterpret_cast<const float4*>(scale + k));
      const float4 sb = __ldg(reinterpret_cast<const float4*>(scale + k + 4));
      *reinterpret_cast<uint4*>(p.xs + (long long)t * p.width + k) =
          make_uint4(pack_bf16x2(a.x * sa.x, a.y * sa.y),
                     pack_bf16x2(a.z * sa.z, a.w * sa.w),
                     pack_bf16x2(b.x * sb.x, b.y * sb.y),
                     pack_bf16x2(b.z * sb.z, b.w * sb.w));
      q = a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b.x * b.x +
          b.y * b.y + b.z * b.z + b.w * b.w;
    }
    q = warp_sum(q);  // per_tok is a multiple of 32: one token per warp
    if (lane == 0 && c < total) atomicAdd(ss + t, q);
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Per-token rstd of the phase's RMSNorm into shared memory.  The sums of
// squares are loaded (`ssv`, issued by the caller before its first batch of
// operand loads so that both round trips overlap) and stored once per CTA:
// read per task from global memory, the whole grid would queue on the few
// L2 lines that hold them.
__device__ __forceinline__ float issue_ss(const Params& p, const float* ss, int wtid) {
  return wtid < TOK ? __ldcg(ss + min(wtid, p.n_tok - 1)) : 0.f;
}
__device__ __forceinline__ void publish_rstd(const Params& p, float ssv, float* s_rstd,
                                             int wtid) {
  if (wtid < TOK) s_rstd[wtid] = rsqrtf(ssv / p.width + p.eps);
  bar128();
}

// hb[t,i] = bf16(gelu(rs*g + bg) * (rs*u + bu)), (g,u) = acc_gu[t, 2i..2i+1],
// rs = rstd of ss_post
__device__ void prep_geglu(const Params& p, const float* gub, const float* ss,
                           float* s_rstd, int wtid) {
  const int per_tok = p.mlp / 8;
  const int total = p.n_tok * per_tok;
  const int ld = 2 * p.mlp;
  constexpr int PB = 2;
  const int stride = gridDim.x * 128;
  float4 q[PB][4];
  auto load = [&](int base) {
#pragma unroll
    for (int u = 0; u < PB; ++u) {
      const int c = base + u * stride;
#pragma unroll
      for (int h = 0; h < 4; ++h) q[u][h] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < total) {
        const int t = c / per_tok, i0 = (c % per_tok) * 8;
        const float* src = p.acc_gu + (long long)t * ld + 2 * i0;
#pragma unroll
        for (int h = 0; h < 4; ++h) q[u][h] = ldcg4(src + 4 * h);
      }
    }
  };
  const int base0 = blockIdx.x * 128 + wtid;
  const float ssv = issue_ss(p, ss, wtid);
  load(base0);
  publish_rstd(p, ssv, s_rstd, wtid);
  for (int base = base0; base < total; base += stride * PB) {
    if (base != base0) load(base);
#pragma unroll
    for (int u = 0; u < PB; ++u) {
      const int c = base + u * stride;
      if (c >= total) break;
      const int t = c / per_tok, i0 = (c % per_tok) * 8;
      const float r = s_rstd[t];
      float y[8];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float g0 = r * q[u][h].x, u0 = r * q[u][h].y;
        float g1 = r * q[u][h].z, u1 = r * q[u][h].w;
        if (gub) {
          const float4 bq = __ldg(reinterpret_cast<const float4*>(gub + 2 * i0 + 4 * h));
          g0 += bq.x; u0 += bq.y; g1 += bq.z; u1 += bq.w;
        }
        y[2 * h] = gelu_tanh_f(g0) * u0;
        y[2 * h + 1] = gelu_tanh_f(g1) * u1;
      }
      *reinterpret_cast<uint4*>(p.hb + (long long)t * p.mlp + i0) =
          make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                     pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// q = rope(rstd*acc_q + b), k = rope(rstd*acc_k + b), v = rstd*acc_v + b for
// the suffix tokens, written once as bf16 for every attention item; rstd of
// ss_in.  Task (t, i): i < (H+1)*hd/2 is a rotary pair of a query head or
// the key head, otherwise a pair (d, d + hd/2) of the value head.
__device__ void finalize_qkv(const Params& p, int layer, const float* ss, float* s_rstd,
                             int wtid) {
  const int H = p.heads, hd = p.hd, half = hd >> 1;
  const int qkv_ld = (H + 2) * hd;
  const int per_tok = (H + 2) * half;
  const int total = p.n_tok * per_tok;
  const float* bias = p.qkv_bias ? p.qkv_bias + (long long)layer * qkv_ld : nullptr;
  constexpr int FB = 4;
  const int stride = gridDim.x * 128;
  float2 a[FB], cs[FB];
  auto load = [&](int base) {
#pragma unroll
    for (int u = 0; u < FB; ++u) {
      const int c = base + u * stride;
      a[u] = cs[u] = make_float2(0.f, 0.f);
      if (c < total) {
        const int t = c / per_tok, i = c % per_tok;
        const float* row = p.acc_qkv + (long long)t * qkv_ld;
        if (i < (H + 1) * half) {
          const int hh = i / half, ii = i % half;
          a[u] = __ldcg(reinterpret_cast<const float2*>(row + hh * hd + 2 * ii));
          cs[u] = __ldg(reinterpret_cast<const float2*>(
              p.rope_suf + ((long long)t * half + ii) * 2));
        } else {
          const int d = i - (H + 1) * half;
          a[u].x = __ldcg(row + (H + 1) * hd + d);
          a[u].y = __ldcg(row + (H + 1) * hd + d + half);
        }
      }
    }
  };
  const int base0 = blockIdx.x * 128 + wtid;
  const float ssv = issue_ss(p, ss, wtid);
  load(base0);
  publish_rstd(p, ssv, s_rstd, wtid);
  for (int base = base0; base < total; base += stride * FB) {
    if (base != base0) load(base);
#pragma unroll
    for (int u = 0; u < FB; ++u) {
      const int c = base + u * stride;
      if (c >= total) break;
      const int t = c / per_tok, i = c % per_tok;
      const float r = s_rstd[t];
      if (i < (H + 1) * half) {
        const int hh = i / half, ii = i % half;
        float x1 = r * a[u].x, x2 = r * a[u].y;
        if (bias) { x1 += bias[hh * hd + 2 * ii]; x2 += bias[hh * hd + 2 * ii + 1]; }
        const float o1 = x1 * cs[u].x - x2 * cs[u].y;
        const float o2 = x2 * cs[u].x + x1 * cs[u].y;
        bf16* dst = hh < H ? p.qb + (long long)t * H * hd + hh * hd
                           : p.kc + layer * p.cache_layer + (long long)(p.n_prefix + t) * hd;
        dst[ii] = __float2bfloat16(o1);
        dst[ii + half] = __float2bfloat16(o2);
      } else {
        const int d = i - (H + 1) * half;
        float v1 = r * a[u].x, v2 = r * a[u].y;
        if (bias) { v1 += bias[(H + 1) * hd + d]; v2 += bias[(H + 1) * hd + d + half]; }
        bf16* dst = p.vc + layer * p.cache_layer + (long long)(p.n_prefix + t) * hd;
        dst[d] = __float2bfloat16(v1);
        dst[d + half] = __float2bfloat16(v2);
      }
    }
  }
  // the attention phase reads q, k and v through TMA (async proxy)
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// merge of the key-block partials of one (head, token) row -> attn (bf16)
constexpr int MAX_NKB = 16;
// merge of the key-block partials: task (head, token, 8 dims), spread over
// the whole grid (one task per thread for the PI0 shapes)
__device__ void merge_partials(const Params& p, int wtid) {
  const int S = p.n_tok, hd = p.hd;
  const int octs = hd / 8;
  const int total = p.heads * S * octs;
  for (int c = blockIdx.x * 128 + wtid; c < total; c += gridDim.x * 128) {
    const int row = c / octs, d = (c % octs) * 8;
    const int h = row / S, t = row % S;
    float2 ml[MAX_NKB];
#pragma unroll
    for (int kb = 0; kb < MAX_NKB; ++kb) {
      ml[kb] = make_float2(-INFINITY, 0.f);
      if (kb < p.nkb)
        ml[kb] = __ldcg(reinterpret_cast<const float2*>(
            p.part_ml + (((long long)h * p.nkb + kb) * TOK + t) * 2));
    }
    uint4 o[MAX_NKB];
#pragma unroll
    for (int kb = 0; kb < MAX_NKB; ++kb) {
      o[kb] = make_uint4(0u, 0u, 0u, 0u);
      if (kb < p.nkb)
        o[kb] = __ldcg(reinterpret_cast<const uint4*>(
            reinterpret_cast<const bf16*>(p.part_o) +
            (((long long)h * p.nkb + kb) * TOK + t) * hd + d));
    }
    float M = -INFINITY;
#pragma unroll
    for (int kb = 0; kb < MAX_NKB; ++kb)
      if (ml[kb].y > 0.f) M = fmaxf(M, ml[kb].x);
    float L = 0.f;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kb = 0; kb < MAX_NKB; ++kb) {
      if (ml[kb].y > 0.f) {
        const float w = exp2f(ml[kb].x - M) * ml[kb].y;  // weight x block sum
        L += w;
        const uint32_t wd[4] = {o[kb].x, o[kb].y, o[kb].z, o[kb].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wd[e]));
          acc[2 * e] += w * f.x;
          acc[2 * e + 1] += w * f.y;
        }
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    *reinterpret_cast<uint4*>(p.attn + (long long)t * p.heads * hd + h * hd + d) =
        make_uint4(pack_bf16x2(acc[0] * inv, acc[1] * inv), pack_bf16x2(acc[2] * inv, acc[3] * inv),
                   pack_bf16x2(acc[4] * inv, acc[5] * inv), pack_bf16x2(acc[6] * inv, acc[7] * inv));
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(THREADS, 1)
    expert_step_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                       const __grid_constant__ CUtensorMap tm_o,
                       const __grid_constant__ CUtensorMap tm_gu,
                       const __grid_constant__ CUtensorMap tm_down,
                       const __grid_constant__ CUtensorMap tb_xs,
                       const __grid_constant__ CUtensorMap tb_attn,
                       const __grid_constant__ CUtensorMap tb_h,
                       const __grid_constant__ CUtensorMap ta_q,
                       const __grid_constant__ CUtensorMap ta_k,
                       const __grid_constant__ CUtensorMap ta_v,
                       const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* region = smem + STAGES * A_BYTES;  // B operand / attention tiles
  uint64_t* full = reinterpret_cast<uint64_t*>(region + REGION_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* b_full = empty + STAGES;
  uint64_t* t_full = b_full + 1;
  uint64_t* t_empty = t_full + 1;
  uint64_t* a_full = t_empty + 1;  // attention operands landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(a_full + 1);
  // per-token rstd of the phase's RMSNorm, loaded once per CTA and phase:
  // read per task from global memory, the whole grid would queue on the
  // few L2 lines that hold the sums of squares
  float* s_rstd = reinterpret_cast<float*>(region + REGION_BYTES + 256);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(b_full, 1);
    mbar_init(t_full, 1);
    mbar_init(t_empty, 4);
    mbar_init(a_full, 1);
    fence_barrier_init();
    prefetch_tensormap(&tm_qkv);
    prefetch_tensormap(&tm_o);
    prefetch_tensormap(&tm_gu);
    prefetch_tensormap(&tm_down);
    prefetch_tensormap(&tb_xs);
    prefetch_tensormap(&tb_attn);
    prefetch_tensormap(&tb_h);
    prefetch_tensormap(&ta_q);
    prefetch_tensormap(&ta_k);
    prefetch_tensormap(&ta_v);
  }
  // An abort flag left raised by an earlier launch on this workspace (one of
  // whose waits gave up) is reported, and the launch then does no work at
  // all (no copy or MMA is issued) instead of returning silently wrong
  // results; the host clears the workspace after reading the status.
  __shared__ int s_skip;
  if (threadIdx.x == 0) {
    s_skip = aborted(p) ? 1 : 0;
    if (s_skip && cta == 0) record_device_error(FVB_ERR_DEVICE_TIMEOUT);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 64);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool skip = s_skip != 0;
  const CUtensorMap* maps[N_GEMM] = {&tm_qkv, &tm_o, &tm_gu, &tm_down};
  // programmatic dependent launch: the next kernel may be scheduled now (it
  // waits for this grid's completion before touching its outputs); the
  // weight producer streams static weights at once, everything that reads
  // activations waits for the previous kernel first
  griddep_launch_dependents();

  if (skip) {
    // nothing issued: straight to the TMEM release
  } else if (warp == 0) {
    // ---- weight producer: every tile of every GEMM item, in order ----
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      int it = 0;
      for (int l = 0; l < p.n_layers; ++l) {
        for (int gi = 0; gi < N_GEMM; ++gi) {
          const Gemm& g = p.g[gi];
          for (int w = cta; w < g.items; w += G) {
            const int mt = w % g.m_tiles, sp = w / g.m_tiles;
            const int kt0 = sp * g.kt_per, kt1 = min(kt0 + g.kt_per, g.k_tiles);
            for (int kt = kt0; kt < kt1; ++kt, ++it) {
              const int s = it % p.stages;
              if (!wait_bar(p, &empty[s], ((it / p.stages) & 1) ^ 1)) goto producer_done;
              mbar_arrive_expect_tx(&full[s], A_BYTES);
              tma_load_2d_stream(ring + s * A_BYTES, maps[gi], kt * 64,
                                 l * g.rows + mt * 128, &full[s], pol);
            }
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(128, TOK);
      int it = 0, j = 0;
      const uint32_t bbase = smem_u32(region);
      for (int l = 0; l < p.n_layers; ++l) {
        for (int gi = 0; gi < N_GEMM; ++gi) {
          const Gemm& g = p.g[gi];
          for (int w = cta; w < g.items; w += G, ++j) {
            const int sp = w / g.m_tiles;
            const int kt0 = sp * g.kt_per, kt1 = min(kt0 + g.kt_per, g.k_tiles);
            if (!wait_bar(p, b_full, j & 1)) goto mma_done;
            if (!wait_bar(p, t_empty, (j & 1) ^ 1)) goto mma_done;
            tc_fence_after();
            for (int kt = kt0; kt < kt1; ++kt, ++it) {
              const int s = it % p.stages;
              if (!wait_bar(p, &full[s], (it / p.stages) & 1)) goto mma_done;
              tc_fence_after();
              const uint64_t da = smem_desc_sw128(smem_u32(ring + s * A_BYTES));
              const uint64_t db = smem_desc_sw128(bbase + (kt - kt0) * BKT_BYTES);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                tc_mma_bf16(tmem, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2),
                            IDESC, (kt > kt0 || kk > 0) ? 1u : 0u);
              tc_commit(&empty[s]);
            }
            tc_commit(t_full);
          }
        }
      }
    mma_done:;
    }
  } else {
    // ---- workers: B builders, epilogues, attention, merges, barriers ----
    griddep_wait();
    const int wtid = threadIdx.x - 64;
    const int q = warp & 3;
    // epilogue transpose stage: [4 warps][16 tokens][32 features + 4]
    float* estage = reinterpret_cast<float*>(region + MAX_KT * BKT_BYTES) +
                    (warp - 2) * 16 * 36;
    const int qkv_ld = (p.heads + 2) * p.hd;
    int j = 0;
    const bool tr = p.trace && wtid == 0 && cta < 256;
    uint32_t a_items = 0;  // attention items run by this CTA (a_full phases)
    if (tr) g_mega_trace[cta][0] = globaltimer_ns();
    for (int l = 0; l < p.n_layers; ++l) {
      // phases: 0 prep QKV operand, 1 QKV, 2 finalize q/k/v, 3 attention,
      // 4 merge, 5 o_proj, 6 prep gate/up operand, 7 gate/up, 8 prep down
      // operand, 9 down
      for (int ph = 0; ph < 10; ++ph) {
        if (ph == 0) {
          // clear the gate/up accumulators and ss_post (read in ph 8 of the
          // previous layer), then x*(1+w_in) and ss_in
          for (int i = cta * 128 + wtid; i < p.n_tok * 2 * p.mlp / 4; i += G * 128)
            reinterpret_cast<float4*>(p.acc_gu)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (cta == 0 && wtid < TOK) p.ss_post[wtid] = 0.f;
          prep_scaled(p, p.in_scale + (long long)l * p.width, p.ss_in, wtid);
        } else if (ph == 2) {
          finalize_qkv(p, l, p.ss_in, s_rstd, wtid);
        } else if (ph == 3) {
          // generic-proxy writes to the region (epilogue staging) before the
          // TMA writes of the attention operands
          fence_async_smem();
          bar128();
          for (int w = cta; w < p.heads * p.nkb; w += G)
            attention_item(p, l, w, region, a_full, (a_items++) & 1, &ta_q, &ta_k, &ta_v,
                           wtid, tr && l == 0 && w == cta);
        } else if (ph == 4) {  // merge; clear the QKV accumulators (read in ph 2)
          merge_partials(p, wtid);
          asm volatile("fence.proxy.async.global;" ::: "memory");
          for (int i = cta * 128 + wtid; i < p.n_tok * qkv_ld / 4; i += G * 128)
            reinterpret_cast<float4*>(p.acc_qkv)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (cta == 0 && wtid < TOK) p.ss_in[wtid] = 0.f;
        } else if (ph == 6) {
          prep_scaled(p, p.post_scale + (long long)l * p.width, p.ss_post, wtid);
        } else if (ph == 8) {
          prep_geglu(p, p.gu_bias ? p.gu_bias + (long long)l * 2 * p.mlp : nullptr,
                     p.ss_post, s_rstd, wtid);
        } else {
          const int gi = ph == 1 ? 0 : (ph == 5 ? 1 : (ph == 7 ? 2 : 3));
          const Gemm& g = p.g[gi];
          const CUtensorMap* bmap = gi == 1 ? &tb_attn : (gi == 3 ? &tb_h : &tb_xs);
          // generic-proxy writes to the region (attention tiles) before the
          // TMA writes of this phase's B operands
          fence_async_smem();
          bar128();
          for (int w = cta; w < g.items; w += G, ++j) {
            const int mt = w % g.m_tiles, sp = w / g.m_tiles;
            const int kt0 = sp * g.kt_per, kt1 = min(kt0 + g.kt_per, g.k_tiles);
            const int nkt = kt1 - kt0;
            // B operand (64 tokens x this K slice) by TMA; the previous
            // item's MMAs have finished reading the region (its epilogue
            // waited for them)
            if (wtid == 0) {
              // the m_tiles CTAs of one K slice read the same B tiles; start
              // each at a different k-tile so their requests spread over L2
              mbar_arrive_expect_tx(b_full, nkt * BKT_BYTES);
              for (int i0 = 0; i0 < nkt; ++i0) {
                const int i = (i0 + mt) % nkt;
                tma_load_2d(region + i * BKT_BYTES, bmap, (kt0 + i) * 64, 0, b_full);
              }
            }
            // the lane that issued goes first: spinning lanes of a diverged
            // warp can otherwise hold it off
            __syncwarp();
            // epilogue: thread = weight row (output feature), 64 token columns
            const bool ok = wait_bar(p, t_full, j & 1);
            __syncwarp();
            if (ok) {
              tc_fence_after();
              float* dst;
              long long ldd;
              float gsc = 1.f;
              const int f = mt * 128 + q * 32 + lane;  // this thread's row
              if (gi == 0) { dst = p.acc_qkv; ldd = qkv_ld; }
              else if (gi == 2) { dst = p.acc_gu; ldd = 2 * p.mlp; }
              else {
                dst = p.x; ldd = p.width;
                const float* gate = gi == 1 ? p.o_gate : p.down_gate;
                if (gate) gsc = __ldg(gate + (long long)l * p.width + f);
              }
              // transpose each 16-token chunk through shared memory so that a
              // lane owns 4 consecutive features of one token: one 16-byte
              // vector reduction instead of four scalar atomics
              const int f0 = mt * 128 + q * 32;
#pragma unroll 1
              for (int c = 0; c < TOK; c += 16) {
                if (c >= p.n_tok) break;
                uint32_t r[16];
                tmem_ld16_sync(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, r);
#pragma unroll
                for (int jj = 0; jj < 16; ++jj)
                  estage[jj * 36 + lane] = gsc * __uint_as_float(r[jj]);
                __syncwarp();
#pragma unroll
                for (int it = 0; it < 4; ++it) {
                  const int jj = it * 4 + (lane >> 3);   // token within chunk
                  const int fq = (lane & 7) * 4;         // 4 features
                  if (c + jj < p.n_tok) {
                    const float4 v = *reinterpret_cast<const float4*>(estage + jj * 36 + fq);
                    float* a = dst + (long long)(c + jj) * ldd + f0 + fq;
                    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(a),
                                 "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                                 : "memory");
                  }
                }
                __syncwarp();
              }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(t_empty);
          }
        }
        if (tr && l == 0) g_mega_trace[cta][1 + 2 * ph] = globaltimer_ns();
        grid_sync(p, wtid);
        if (tr && l == 0) g_mega_trace[cta][2 + 2 * ph] = globaltimer_ns();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

}  // namespace mega
}  // namespace fvb
