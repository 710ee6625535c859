// Persistent expert-layer kernel for the denoise loop: all layers of one
// flow-matching step (action-expert Gemma stack over <= 64 suffix tokens) in
// one cooperative launch, one CTA per SM.
//
// Per layer, six phases separated by grid barriers:
//   P1 QKV   acc_qkv[t,f] += W_qkv[f,k] * (x[t,k](1+w_in[k]))  (split-K, f32
//            atomics); the row-tile-0 items also add sum_k x^2 into ss_in[t]
//   P2 ATT   per (head, 64-key block): q,k,v = rope(rstd_in[t]*acc + bias),
//            masked attention over prefix cache keys + suffix keys -> partial
//   P3 CMB   merge the key-block partials -> attn[t, h*hd + d] (bf16)
//   P4 O     x[t,f] += gate_o[f] * (W_o attn)  (split-K atomics)
//   P5 GU    acc_gu[t,f] += W_gu[f,k] * (x[t,k](1+w_post[k])), ss_post[t]
//   P6 DOWN  x[t,f] += gate_d[f] * (W_down gelu(g)*u), with
//            g,u = rstd_post[t]*acc_gu + bias built into the MMA's B operand
// RMSNorm is linear in the un-normalised row apart from the per-token factor
// rstd, so the GEMM runs on x*(1+w) and rstd is applied by the consumer; for
// adaRMSNorm the shift enters as W*shift, precomputed per step (bias arrays).
//
// Roles: warp 0 lane 0 streams every weight tile of the step through a
// STAGES-deep TMA ring in a fixed order and never waits for a barrier (the
// weights do not depend on the previous phase); warp 1 lane 0 issues
// tcgen05.mma (M=128 weight rows, N=64 tokens, K=16) into a 64-column TMEM
// accumulator; warps 2..5 build the B operand (tokens x K-slice, bf16, 128-byte
// swizzle) in shared memory, run the epilogue atomics, the attention and the
// merge, and take part in the grid barriers.
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
constexpr int APITCH = 264;                // attention smem row pitch (bf16)
constexpr int ATILE = 64 * APITCH;         // elements per attention tile
constexpr int REGION_BYTES = 3 * ATILE * 2 + 64 + 64 * 4;  // >= MAX_KT*BKT
constexpr int SMEM_BYTES = 1024 + STAGES * A_BYTES + REGION_BYTES + 256;
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
  const bf16* kc;           // [L, cache_rows, hd]
  const bf16* vc;
  long long cache_layer;    // elements per layer of the cache
  const uint8_t* key_valid;
  const int* blocks;
  const int* positions;
  const float* rope_cs;
  float scale_log2;
  // workspace
  float* acc_qkv;  // [TOK, (H+2)*hd]
  float* acc_gu;   // [TOK, 2*mlp]
  float* ss_in;    // [TOK]
  float* ss_post;  // [TOK]
  float* part_o;   // [heads*nkb, TOK, hd]
  float* part_ml;  // [heads*nkb, TOK, 2]
  bf16* attn;      // [TOK, heads*hd]
  unsigned* bar;   // [0] count, [1] generation, [2] abort
  int nkb;         // key blocks of 64
};

// ---------------------------------------------------------------------------
// waits with a time limit and a shared abort flag
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool aborted(const Params& p) {
  return *reinterpret_cast<volatile unsigned*>(p.bar + 2) != 0u;
}

__device__ __forceinline__ void set_abort(const Params& p) {
  record_device_error(FVB_ERR_DEVICE_TIMEOUT);
  atomicExch(p.bar + 2, 1u);
}

__device__ __forceinline__ bool wait_bar(const Params& p, uint64_t* bar,
                                         uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(addr, parity)) return true;
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

// Grid barrier among the 4 worker warps of every CTA.
__device__ __forceinline__ void grid_sync(const Params& p, int wtid) {
  __threadfence();
  bar128();
  if (wtid == 0) {
    volatile unsigned* gen = p.bar + 1;
    const unsigned g = *gen;
    if (atomicAdd(p.bar, 1u) == gridDim.x - 1) {
      p.bar[0] = 0u;
      __threadfence();
      atomicAdd(p.bar + 1, 1u);
    } else {
      const uint64_t t0 = globaltimer_ns();
      while (*gen == g) {
        if (aborted(p)) break;
        if (globaltimer_ns() - t0 > FVB_WAIT_LIMIT_NS) {
          set_abort(p);
          break;
        }
      }
    }
    __threadfence();
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
// B operand builders (worker warps, 128 threads)
// ---------------------------------------------------------------------------
// The builders walk 16-byte B chunks (token t, 8 consecutive k) with the
// chunk index fastest along k, four chunks per thread per round: the global
// loads of a round are all issued before any of them is used.
constexpr int BATCH = 4;

// B[t,k] = x[t,k]*scale[k] for k in [k0, k0 + nkt*64); optional sum of x^2
__device__ void build_b_scaled(const Params& p, uint8_t* B, const float* x,
                               int ldx, const float* scale, int k0, int nkt,
                               float* ss, int wtid) {
  const int nch = nkt * 8, total = TOK * nch;
  for (int base = wtid; base < total; base += 128 * BATCH) {
    float4 a[BATCH], b[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int c = base + u * 128;
      const int t = c / nch, kc = c % nch;
      a[u] = b[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < total && t < p.n_tok) {
        const float* src = x + (long long)t * ldx + k0 + kc * 8;
        a[u] = ldcg4(src);
        b[u] = ldcg4(src + 4);
      }
    }
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int c = base + u * 128;
      if (c >= total) break;
      const int t = c / nch, kc = c % nch;
      uint4 w = make_uint4(0, 0, 0, 0);
      if (t < p.n_tok) {
        const int k = k0 + kc * 8;
        const float4 sa = __ldg(reinterpret_cast<const float4*>(scale + k));
        const float4 sb = __ldg(reinterpret_cast<const float4*>(scale + k + 4));
        w = make_uint4(pack_bf16x2(a[u].x * sa.x, a[u].y * sa.y),
                       pack_bf16x2(a[u].z * sa.z, a[u].w * sa.w),
                       pack_bf16x2(b[u].x * sb.x, b[u].y * sb.y),
                       pack_bf16x2(b[u].z * sb.z, b[u].w * sb.w));
        if (ss) {
          const float q = a[u].x * a[u].x + a[u].y * a[u].y + a[u].z * a[u].z +
                          a[u].w * a[u].w + b[u].x * b[u].x + b[u].y * b[u].y +
                          b[u].z * b[u].z + b[u].w * b[u].w;
          atomicAdd(ss + t, q);
        }
      }
      *reinterpret_cast<uint4*>(B + b_off(t, kc)) = w;
    }
  }
}

// B[t,k] = attn[t,k] (bf16 copy)
__device__ void build_b_copy(const Params& p, uint8_t* B, const bf16* src,
                             int lds, int k0, int nkt, int wtid) {
  const int nch = nkt * 8, total = TOK * nch;
  for (int base = wtid; base < total; base += 128 * BATCH) {
    uint4 w[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int c = base + u * 128;
      const int t = c / nch, kc = c % nch;
      w[u] = make_uint4(0, 0, 0, 0);
      if (c < total && t < p.n_tok)
        w[u] = __ldcg(reinterpret_cast<const uint4*>(src + (long long)t * lds + k0 + kc * 8));
    }
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int c = base + u * 128;
      if (c >= total) break;
      *reinterpret_cast<uint4*>(B + b_off(c / nch, c % nch)) = w[u];
    }
  }
}

// B[t,i] = gelu(rs*g + bg) * (rs*u + bu), (g, u) = acc_gu[t, 2i], [t, 2i+1]
__device__ void build_b_geglu(const Params& p, uint8_t* B, const float* gub,
                              int k0, int nkt, int wtid) {
  const int nch = nkt * 8, total = TOK * nch;
  const int ld = 2 * p.mlp;
  for (int base = wtid; base < total; base += 128 * 2) {
    float4 q[2][4];
    float rs[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = base + u * 128;
      const int t = c / nch, kc = c % nch;
      rs[u] = 0.f;
#pragma unroll
      for (int h = 0; h < 4; ++h) q[u][h] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < total && t < p.n_tok) {
        rs[u] = __ldcg(p.ss_post + t);
        const float* src = p.acc_gu + (long long)t * ld + 2 * (k0 + kc * 8);
#pragma unroll
        for (int h = 0; h < 4; ++h) q[u][h] = ldcg4(src + 4 * h);
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = base + u * 128;
      if (c >= total) break;
      const int t = c / nch, kc = c % nch;
      uint4 w = make_uint4(0, 0, 0, 0);
      if (t < p.n_tok) {
        const float r = rsqrtf(rs[u] / p.width + p.eps);
        const int i0 = k0 + kc * 8;
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
        w = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                       pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
      }
      *reinterpret_cast<uint4*>(B + b_off(t, kc)) = w;
    }
  }
}

// ---------------------------------------------------------------------------
// attention block: 64 query rows (one head) x one 64-key block
// ---------------------------------------------------------------------------
__device__ void attention_item(const Params& p, int layer, int item,
                               uint8_t* region, int wtid) {
  const int H = p.heads, hd = p.hd, half = hd >> 1;
  const int h = item / p.nkb, kb = item % p.nkb;
  const int S = p.n_tok, E = p.n_prefix, n_kv = E + S;
  const int qkv_ld = (H + 2) * hd;
  bf16* sQ = reinterpret_cast<bf16*>(region);
  bf16* sK = sQ + ATILE;
  bf16* sV = sK + ATILE;
  uint8_t* sMask = reinterpret_cast<uint8_t*>(sV + ATILE);
  int* sKb = reinterpret_cast<int*>(sMask + 64);
  const float* bias = p.qkv_bias ? p.qkv_bias + (long long)layer * qkv_ld : nullptr;
  const bf16* kc = p.kc + layer * p.cache_layer;
  const bf16* vc = p.vc + layer * p.cache_layer;

  // prefix keys of this block: cp.async from the bf16 cache
  const int key0 = kb * 64;
  for (int c = wtid; c < 64 * (hd / 8); c += 128) {
    const int r = c / (hd / 8), cc = c % (hd / 8);
    const int key = key0 + r;
    // rows past the prefix are written by the suffix build below (no async
    // copy may target them)
    if (key < E) {
      cp_async16(sK + r * APITCH + cc * 8, kc + (long long)key * hd + cc * 8, true);
      cp_async16(sV + r * APITCH + cc * 8, vc + (long long)key * hd + cc * 8, true);
    }
  }
  cp_async_commit();
  // queries (and the suffix keys/values of this block) from the QKV
  // accumulator: rows t x rotary pairs i, four per thread per round
  for (int base = wtid; base < 64 * half; base += 128 * BATCH) {
    float2 a[BATCH], cs[BATCH];
    float rs[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int c = base + u * 128;
      const int t = c / half, i = c % half;
      a[u] = cs[u] = make_float2(0.f, 0.f);
      rs[u] = 0.f;
      if (c < 64 * half && t < S) {
        rs[u] = __ldcg(p.ss_in + t);
        a[u] = __ldcg(reinterpret_cast<const float2*>(
            p.acc_qkv + (long long)t * qkv_ld + h * hd + 2 * i));
        cs[u] = *reinterpret_cast<const float2*>(
            p.rope_cs + ((long long)p.positions[t] * half + i) * 2);
      }
    }
#pragma unroll
    for (int u = 0; u < BATCH; ++u) {
      const int c = base + u * 128;
      if (c >= 64 * half) break;
      const int t = c / half, i = c % half;
      float q1 = 0.f, q2 = 0.f;
      if (t < S) {
        const float r = rsqrtf(rs[u] / p.width + p.eps);
        float x1 = r * a[u].x, x2 = r * a[u].y;
        if (bias) { x1 += bias[h * hd + 2 * i]; x2 += bias[h * hd + 2 * i + 1]; }
        q1 = x1 * cs[u].x - x2 * cs[u].y;
        q2 = x2 * cs[u].x + x1 * cs[u].y;
      }
      sQ[t * APITCH + i] = __float2bfloat16(q1);
      sQ[t * APITCH + i + half] = __float2bfloat16(q2);
    }
  }
  const int r_suf = max(0, E - key0);  // first row of this block past the prefix
  if (r_suf < 64) {
    const int nrow = 64 - r_suf;
    for (int base = wtid; base < nrow * half; base += 128 * BATCH) {
      float2 a[BATCH], cs[BATCH];
      float vv[BATCH][2], rs[BATCH];
#pragma unroll
      for (int u = 0; u < BATCH; ++u) {
        const int c = base + u * 128;
        const int r = r_suf + c / half, i = c % half;
        const int key = key0 + r;
        a[u] = cs[u] = make_float2(0.f, 0.f);
        vv[u][0] = vv[u][1] = rs[u] = 0.f;
        if (c < nrow * half && key < n_kv) {
          const int s = key - E;
          const float* row = p.acc_qkv + (long long)s * qkv_ld;
          rs[u] = __ldcg(p.ss_in + s);
          a[u] = __ldcg(reinterpret_cast<const float2*>(row + H * hd + 2 * i));
          vv[u][0] = __ldcg(row + (H + 1) * hd + i);
          vv[u][1] = __ldcg(row + (H + 1) * hd + i + half);
          cs[u] = *reinterpret_cast<const float2*>(
              p.rope_cs + ((long long)p.positions[s] * half + i) * 2);
        }
      }
#pragma unroll
      for (int u = 0; u < BATCH; ++u) {
        const int c = base + u * 128;
        if (c >= nrow * half) break;
        const int r = r_suf + c / half, i = c % half;
        float k1 = 0.f, k2 = 0.f, v1 = 0.f, v2 = 0.f;
        if (key0 + r < n_kv) {
          const float rr = rsqrtf(rs[u] / p.width + p.eps);
          float x1 = rr * a[u].x, x2 = rr * a[u].y;
          v1 = rr * vv[u][0];
          v2 = rr * vv[u][1];
          if (bias) {
            x1 += bias[H * hd + 2 * i]; x2 += bias[H * hd + 2 * i + 1];
            v1 += bias[(H + 1) * hd + i]; v2 += bias[(H + 1) * hd + i + half];
          }
          k1 = x1 * cs[u].x - x2 * cs[u].y;
          k2 = x2 * cs[u].x + x1 * cs[u].y;
        }
        sK[r * APITCH + i] = __float2bfloat16(k1);
        sK[r * APITCH + i + half] = __float2bfloat16(k2);
        sV[r * APITCH + i] = __float2bfloat16(v1);
        sV[r * APITCH + i + half] = __float2bfloat16(v2);
      }
    }
  }
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
  cp_async_wait<0>();
  bar128();

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
    ldsm_x4(sQa + ((warp * 16 + (lane & 15)) * APITCH + kk * 16 + (lane >> 4) * 8) * 2,
            a0, a1, a2, a3);
#pragma unroll
    for (int nt = 0; nt < 8; nt += 2) {
      uint32_t b0, b1, b2, b3;
      const int mi = lane >> 3, rr = lane & 7;
      const int key = nt * 8 + (mi >> 1) * 8 + rr;
      ldsm_x4(sKa + (key * APITCH + kk * 16 + (mi & 1) * 8) * 2, b0, b1, b2, b3);
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
  float* po = p.part_o + (long long)item * TOK * hd;
  float* pml = p.part_ml + (long long)item * TOK * 2;
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
        ldsm_x4_t(sVa + (key * APITCH + col) * 2, b0, b1, b2, b3);
        mma_bf16_16816(o[nt], a0, a1, a2, a3, b0, b1);
        mma_bf16_16816(o[nt + 1], a0, a1, a2, a3, b2, b3);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int d = dp * 64 + nt * 8 + (lane & 3) * 2;
      if (r0 < S)
        __stcg(reinterpret_cast<float2*>(po + (long long)r0 * hd + d),
               make_float2(o[nt][0], o[nt][1]));
      if (r1 < S)
        __stcg(reinterpret_cast<float2*>(po + (long long)r1 * hd + d),
               make_float2(o[nt][2], o[nt][3]));
    }
  }
  if ((lane & 3) == 0) {
    if (r0 < S) __stcg(reinterpret_cast<float2*>(pml + r0 * 2), make_float2(mx0, l0));
    if (r1 < S) __stcg(reinterpret_cast<float2*>(pml + r1 * 2), make_float2(mx1, l1));
  }
  bar128();  // the region is reused by the next item
}

// merge of the key-block partials of one (head, token) row -> attn (bf16)
__device__ void combine_row(const Params& p, int row, int wtid) {
  const int S = p.n_tok, hd = p.hd;
  const int h = row / S, t = row % S;
  float M = -INFINITY;
  for (int kb = 0; kb < p.nkb; ++kb) {
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(
        p.part_ml + ((long long)(h * p.nkb + kb) * TOK + t) * 2));
    if (ml.y > 0.f) M = fmaxf(M, ml.x);
  }
  float L = 0.f, acc0 = 0.f, acc1 = 0.f;
  const int d = wtid * 2;
  for (int kb = 0; kb < p.nkb; ++kb) {
    const long long it = h * p.nkb + kb;
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(p.part_ml + (it * TOK + t) * 2));
    if (ml.y > 0.f) {
      const float w = exp2f(ml.x - M);
      L += w * ml.y;
      const float2 o = __ldcg(reinterpret_cast<const float2*>(p.part_o + (it * TOK + t) * hd + d));
      acc0 += w * o.x;
      acc1 += w * o.y;
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  *reinterpret_cast<uint32_t*>(p.attn + (long long)t * p.heads * hd + h * hd + d) =
      pack_bf16x2(acc0 * inv, acc1 * inv);
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(THREADS, 1)
    expert_step_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                       const __grid_constant__ CUtensorMap tm_o,
                       const __grid_constant__ CUtensorMap tm_gu,
                       const __grid_constant__ CUtensorMap tm_down,
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
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(t_empty + 1);

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
    fence_barrier_init();
    prefetch_tensormap(&tm_qkv);
    prefetch_tensormap(&tm_o);
    prefetch_tensormap(&tm_gu);
    prefetch_tensormap(&tm_down);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 64);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const CUtensorMap* maps[N_GEMM] = {&tm_qkv, &tm_o, &tm_gu, &tm_down};

  if (warp == 0) {
    // ---- weight producer: every tile of every GEMM item, in order ----
    if (lane == 0) {
      int it = 0;
      for (int l = 0; l < p.n_layers; ++l) {
        for (int gi = 0; gi < N_GEMM; ++gi) {
          const Gemm& g = p.g[gi];
          for (int w = cta; w < g.items; w += G) {
            const int mt = w % g.m_tiles, sp = w / g.m_tiles;
            const int kt0 = sp * g.kt_per, kt1 = min(kt0 + g.kt_per, g.k_tiles);
            for (int kt = kt0; kt < kt1; ++kt, ++it) {
              const int s = it % STAGES;
              if (!wait_bar(p, &empty[s], ((it / STAGES) & 1) ^ 1)) goto producer_done;
              mbar_arrive_expect_tx(&full[s], A_BYTES);
              tma_load_2d(ring + s * A_BYTES, maps[gi], kt * 64,
                          l * g.rows + mt * 128, &full[s]);
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
              const int s = it % STAGES;
              if (!wait_bar(p, &full[s], (it / STAGES) & 1)) goto mma_done;
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
    const int wtid = threadIdx.x - 64;
    const int q = warp & 3;
    const int qkv_ld = (p.heads + 2) * p.hd;
    int j = 0;
    for (int l = 0; l < p.n_layers; ++l) {
      for (int ph = 0; ph < 6; ++ph) {
        if (ph == 1) {  // attention
          for (int w = cta; w < p.heads * p.nkb; w += G)
            attention_item(p, l, w, region, wtid);
        } else if (ph == 2) {  // merge; clear the QKV accumulators (read in ph 1)
          for (int r = cta; r < p.heads * p.n_tok; r += G) combine_row(p, r, wtid);
          for (int i = cta * 128 + wtid; i < TOK * qkv_ld; i += G * 128)
            p.acc_qkv[i] = 0.f;
          if (cta == 0 && wtid < TOK) p.ss_in[wtid] = 0.f;
        } else {
          const int gi = ph == 0 ? 0 : ph - 2;  // 0 QKV, 3 O, 4 GU, 5 DOWN
          const Gemm& g = p.g[gi];
          if (ph == 0) {  // clear the gate/up accumulators (read in ph 5)
            for (int i = cta * 128 + wtid; i < TOK * 2 * p.mlp; i += G * 128)
              p.acc_gu[i] = 0.f;
            if (cta == 0 && wtid < TOK) p.ss_post[wtid] = 0.f;
            // ... which must be complete before any item of this phase
            // starts accumulating ss_in (ss_post is cleared here, ss_in in ph 2)
          }
          for (int w = cta; w < g.items; w += G, ++j) {
            const int mt = w % g.m_tiles, sp = w / g.m_tiles;
            const int kt0 = sp * g.kt_per, kt1 = min(kt0 + g.kt_per, g.k_tiles);
            const int nkt = kt1 - kt0;
            // the previous item's MMAs have finished reading the B region
            // (its epilogue waited for them); build this item's B
            if (gi == 0)
              build_b_scaled(p, region, p.x, p.width, p.in_scale + (long long)l * p.width,
                             kt0 * 64, nkt, mt == 0 ? p.ss_in : nullptr, wtid);
            else if (gi == 1)
              build_b_copy(p, region, p.attn, p.heads * p.hd, kt0 * 64, nkt, wtid);
            else if (gi == 2)
              build_b_scaled(p, region, p.x, p.width, p.post_scale + (long long)l * p.width,
                             kt0 * 64, nkt, mt == 0 ? p.ss_post : nullptr, wtid);
            else
              build_b_geglu(p, region, p.gu_bias ? p.gu_bias + (long long)l * 2 * p.mlp : nullptr,
                            kt0 * 64, nkt, wtid);
            fence_async_smem();
            bar128();
            if (wtid == 0) mbar_arrive(b_full);
            // epilogue: thread = weight row (output feature), 64 token columns
            const bool ok = wait_bar(p, t_full, j & 1);
            __syncwarp();
            if (ok) {
              tc_fence_after();
              const int f = mt * 128 + q * 32 + lane;
              float* dst;
              long long ldd;
              float gsc = 1.f;
              if (gi == 0) { dst = p.acc_qkv; ldd = qkv_ld; }
              else if (gi == 2) { dst = p.acc_gu; ldd = 2 * p.mlp; }
              else {
                dst = p.x; ldd = p.width;
                const float* gate = gi == 1 ? p.o_gate : p.down_gate;
                if (gate) gsc = __ldg(gate + (long long)l * p.width + f);
              }
#pragma unroll 1
              for (int c = 0; c < TOK; c += 16) {
                uint32_t r[16];
                tmem_ld16_sync(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, r);
#pragma unroll
                for (int jj = 0; jj < 16; ++jj)
                  if (c + jj < p.n_tok)
                    atomicAdd(dst + (long long)(c + jj) * ldd + f, gsc * __uint_as_float(r[jj]));
              }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(t_empty);
          }
        }
        grid_sync(p, wtid);
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
