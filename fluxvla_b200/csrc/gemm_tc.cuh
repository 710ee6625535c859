// tcgen05 / TMEM tensor-core GEMM for sm_100a:  C[M,N] = A[M,K] * B[N,K]^T.
//
// Persistent: one CTA per SM walks the 128 x BN output tiles (and K splits)
// with a grid-stride loop; tile index = m-tile fastest, so the CTAs running
// at the same time share the same B (weight) tile in the normal orientation
// and stream consecutive weight tiles in the swapped one.
//   warp 0 (one lane)  : TMA producer, STAGES-deep ring of (A,B) k-tiles
//                        (64 bf16 = 128 B per row, 128-byte swizzle)
//   warp 1             : allocates 2*BN TMEM columns (two accumulators); one
//                        lane issues tcgen05.mma (M=128, N=BN, K=16) x4 per
//                        k-tile and commits stages back to the producer
//   warps 2..5         : epilogue; warp w reads TMEM lanes 32*(w%4)..+31
//                        (one accumulator row per thread) with tcgen05.ld.
// The two accumulators let the epilogue of tile j run while the MMA warp
// accumulates tile j+1.
//
// Programmatic dependent launch: the producer issues the weight half of its
// first STAGES k-tiles, then griddepcontrol.wait, then the activation half,
// so weight streaming overlaps the previous kernel's tail.
//
// The epilogue works on (token, feature) pairs: in the normal orientation A
// rows are tokens and B rows are features; with SWAP the A rows are features
// (the weight matrix streams through the M side) and the B rows are tokens,
// which is how the denoise loop runs its 50/51-token GEMMs on tensor cores.
// In the normal orientation each warp stages 32 rows x 32 columns in shared
// memory and writes them back row-contiguous, so every store instruction
// covers whole 32-byte sectors of a few rows; in the swapped orientation
// consecutive lanes already hold consecutive features of one token.
// The epilogue kind and orientation are template parameters, so each kernel
// instantiation carries only its own epilogue code.
#pragma once

#include "common.cuh"

namespace fvb {

struct GemmDev {
  int m, n, k;
  int act;
  int k_tiles, kt_per_split, split;
  int m_tiles, n_tiles, n_work;
  void* out;
  long long ldo;
  const float* bias;
  const float* gate;
  float alpha;
  const bf16* row_add;
  int row_add_mod;
  bf16* k_out;
  bf16* v_out;
  long long ld_kv;
  int n_heads, head_dim;
  const float* rope_cs;
  const int* positions;
  // split-K fixup of swapped non-additive epilogues: f32 partial tiles
  // [m_tiles*n_tiles][BN tokens][128 features] and one arrival counter per
  // tile; all zero between launches (the last CTA of a tile re-zeroes both)
  float* ws;
  unsigned* ws_cnt;
  int trace;  // diagnostics: record per-CTA phase times in g_gemm_trace
  int tma_out;  // normal orientation: the epilogue writes through the output
                // tensor map (TMA store, or TMA f32 reduce-add for F32_ACC)
  // fused norm of the finished f32 output rows (norm_out != null)
  bf16* norm_out;
  long long ld_norm_out;
  const bf16* norm_w;
  const bf16* norm_b;
  float norm_eps;
  int norm_mode;
  unsigned long long* norm_sync;
  // bf16 epilogue: per-element residual and gate (bf16 [m, ld]) or null
  const bf16* res;
  long long ld_res;
  const bf16* gate_tok;
  long long ld_gate_tok;
  int rope_interleaved;  // QKV: store rotary pairs adjacent
};

// Arrivals of one launch at the fused-norm grid barrier add up to exactly
// NORM_SYNC_UNIT (CTA 0 adds the part of the unit that the grid does not
// fill), so the counter is shared by calls of any grid size.
constexpr unsigned long long NORM_SYNC_UNIT = 4096;

// Normalise one row of `dim` (<= 2048, multiple of 128) f32 values into
// bf16: GEMMA_RMS x*rstd*(1+w) or LAYER (x-mean)*rstd*w + b.  One warp; the
// row is read with L2 loads (written by other CTAs' TMA reductions).
__device__ __forceinline__ void norm_row_warp(int mode, const float* xr, bf16* yr,
                                              int dim, const bf16* w,
                                              const bf16* b, float eps,
                                              int lane) {
  const int nv = dim >> 7;
  float4 v[16];
  float s = 0.f, ss = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < nv) v[i] = __ldcg(reinterpret_cast<const float4*>(xr + (i * 32 + lane) * 4));
    s += v[i].x + v[i].y + v[i].z + v[i].w;
    ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  }
  float mean = 0.f, rstd;
  if (mode == FVB_NORM_LAYER) {
    mean = warp_sum(s) / dim;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < nv)
        q += (v[i].x - mean) * (v[i].x - mean) + (v[i].y - mean) * (v[i].y - mean) +
             (v[i].z - mean) * (v[i].z - mean) + (v[i].w - mean) * (v[i].w - mean);
    rstd = rsqrtf(warp_sum(q) / dim + eps);
  } else {
    rstd = rsqrtf(warp_sum(ss) / dim + eps);
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (i >= nv) break;
    const int c0 = (i * 32 + lane) * 4;
    const uint2 wq = *reinterpret_cast<const uint2*>(w + c0);
    const float2 w01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wq.x));
    const float2 w23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wq.y));
    float y0 = (v[i].x - mean) * rstd, y1 = (v[i].y - mean) * rstd;
    float y2 = (v[i].z - mean) * rstd, y3 = (v[i].w - mean) * rstd;
    if (mode == FVB_NORM_LAYER) {
      const uint2 bq = *reinterpret_cast<const uint2*>(b + c0);
      const float2 b01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bq.x));
      const float2 b23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bq.y));
      y0 = y0 * w01.x + b01.x; y1 = y1 * w01.y + b01.y;
      y2 = y2 * w23.x + b23.x; y3 = y3 * w23.y + b23.y;
    } else {
      y0 *= 1.f + w01.x; y1 *= 1.f + w01.y; y2 *= 1.f + w23.x; y3 *= 1.f + w23.y;
    }
    *reinterpret_cast<uint2*>(yr + c0) = make_uint2(pack_bf16x2(y0, y1), pack_bf16x2(y2, y3));
  }
}

__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Diagnostics: per-CTA globaltimer stamps [start, setup done, first weight
// TMA issued, first k-tile landed, last MMA committed, first accumulator
// ready, last epilogue done, end] for the first GEMM_TRACE_CTAS CTAs of a
// launch made with tracing on.
constexpr int GEMM_TRACE_CTAS = 1024;
__device__ unsigned long long g_gemm_trace[GEMM_TRACE_CTAS][16];

__device__ __forceinline__ void trace_stamp(const GemmDev& p, int slot) {
  if (p.trace && blockIdx.x < GEMM_TRACE_CTAS)
    g_gemm_trace[blockIdx.x][slot] = globaltimer_ns();
}

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 192;
constexpr int STAGE_PITCH = 33;  // 32-bit words per staged row

template <int ACT>
__device__ __forceinline__ float apply_act(float x) {
  if (ACT == FVB_ACT_GELU_TANH) return gelu_tanh_f(x);
  if (ACT == FVB_ACT_SILU) return silu_f(x);
  return x;
}

struct Tile {
  int m0, nt, kt0, kt1, split;
};

__device__ __forceinline__ Tile decode_tile(const GemmDev& p, int w) {
  Tile t;
  const int mt = w % p.m_tiles;
  const int rest = w / p.m_tiles;
  t.nt = rest % p.n_tiles;
  t.split = rest / p.n_tiles;
  t.m0 = mt * GEMM_BM;
  t.kt0 = t.split * p.kt_per_split;
  t.kt1 = min(t.kt0 + p.kt_per_split, p.k_tiles);
  return t;
}

__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }

// Cooperative write-back of a warp's staged block of 32 rows x NW 32-bit
// words.  Each lane moves 4 words (16 bytes), so one instruction covers
// 128/NW rows.  All loads (staged words, destination or row_add operands) are
// issued before any store so their latencies overlap.  Words >= NW/2 of a
// row go hi_extra words further (the two rotary halves of a head).
//   MODE 0: store, 1: add to an f32 destination, 2: atomic add (split-K),
//   3: f32 store + bf16 row_add (position embedding)
template <int NW, int MODE, typename DstFn>
__device__ __forceinline__ void warp_writeback(
    const uint32_t* stage, int lane, int rows_valid, int words_valid,
    DstFn dst_of_row, int hi_extra = 0, const bf16* ra_base = nullptr,
    int ra_mod = 1, int ra_ld = 0, int t_base = 0) {
  constexpr int LPR = NW / 4;     // lanes per row
  constexpr int RPI = 32 / LPR;   // rows per instruction
  constexpr int ITER = 32 / RPI;
  const int sub = lane % LPR, rr = lane / LPR;
  const int w0 = sub * 4;
  const int extra = (w0 >= NW / 2) ? hi_extra : 0;
  const bool vec = w0 + 4 <= words_valid;
  float val[ITER][4];
#pragma unroll
  for (int it = 0; it < ITER; ++it) {
    const int row = it * RPI + rr;
    const uint32_t* s = stage + row * STAGE_PITCH + w0;
#pragma unroll
    for (int w = 0; w < 4; ++w) val[it][w] = u2f(s[w]);
    if (row < rows_valid && (MODE == 1 || MODE == 3)) {
      if (MODE == 1) {
        const float* d = reinterpret_cast<const float*>(dst_of_row(row) + w0 + extra);
        if (vec) {
          const float4 o = *reinterpret_cast<const float4*>(d);
          val[it][0] += o.x; val[it][1] += o.y; val[it][2] += o.z; val[it][3] += o.w;
        } else {
#pragma unroll
          for (int w = 0; w < 4; ++w)
            if (w0 + w < words_valid) val[it][w] += d[w];
        }
      } else {
        const bf16* ra = ra_base + (long long)((t_base + row) % ra_mod) * ra_ld + w0;
#pragma unroll
        for (int w = 0; w < 4; ++w)
          if (w0 + w < words_valid) val[it][w] += __bfloat162float(ra[w]);
      }
    }
  }
#pragma unroll
  for (int it = 0; it < ITER; ++it) {
    const int row = it * RPI + rr;
    if (row >= rows_valid) continue;
    uint32_t* d = dst_of_row(row) + w0 + extra;
    if (MODE == 2) {
      if (vec) {
        asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(d),
                     "f"(val[it][0]), "f"(val[it][1]), "f"(val[it][2]),
                     "f"(val[it][3])
                     : "memory");
      } else {
#pragma unroll
        for (int w = 0; w < 4; ++w)
          if (w0 + w < words_valid) atomicAdd(reinterpret_cast<float*>(d) + w, val[it][w]);
      }
    } else if (vec) {
      *reinterpret_cast<uint4*>(d) =
          make_uint4(__float_as_uint(val[it][0]), __float_as_uint(val[it][1]),
                     __float_as_uint(val[it][2]), __float_as_uint(val[it][3]));
    } else {
#pragma unroll
      for (int w = 0; w < 4; ++w)
        if (w0 + w < words_valid) d[w] = __float_as_uint(val[it][w]);
    }
  }
}

// Operands of one tile's epilogue that do not depend on the accumulator,
// loaded before the accumulator is ready (while the MMA warp still runs).
struct EpiPre {
  float fb, fg;            // swap: this feature row's bias and gate*alpha
  int pos;                 // normal QKV: this token row's position
  float x0[16], y0[16];    // first chunk's gathered operands
};

template <int BN, int EPI>
__device__ __forceinline__ void load_rope32(const GemmDev& p, int pos, int f0,
                                            float (&cs)[32]) {
  const int hd = p.head_dim, half = hd >> 1;
  const int i0 = (f0 % hd) >> 1;
  const float4* src =
      reinterpret_cast<const float4*>(p.rope_cs + ((long long)pos * half + i0) * 2);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 q = src[j];
    cs[4 * j] = q.x; cs[4 * j + 1] = q.y; cs[4 * j + 2] = q.z; cs[4 * j + 3] = q.w;
  }
}

// Swapped orientation: chunk operands of 16 tokens (rotary cos/sin for query
// and key rows, the old residual for an unsplit F32_ACC, row_add values).
template <int EPI>
__device__ __forceinline__ void swap_chunk_operands(const GemmDev& p, int fs,
                                                    bool is_qk, int pair_i,
                                                    int t0, float (&x)[16],
                                                    float (&y)[16]) {
  const int n_tok = p.n, n_feat = p.m;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int tt = min(t0 + j, n_tok - 1);
    x[j] = 0.f;
    y[j] = 0.f;
    if (EPI == FVB_EPI_F32_STORE) {
      if (p.row_add)
        x[j] = __bfloat162float(p.row_add[(long long)(tt % p.row_add_mod) * n_feat + fs]);
    } else if (EPI == FVB_EPI_F32_ACC) {
      if (p.split == 1)
        x[j] = reinterpret_cast<const float*>(p.out)[(long long)tt * p.ldo + fs];
    } else if (EPI == FVB_EPI_QKV_ROPE) {
      if (is_qk) {
        const float2 q = *reinterpret_cast<const float2*>(
            p.rope_cs + ((long long)p.positions[tt] * (p.head_dim >> 1) + pair_i) * 2);
        x[j] = q.x;
        y[j] = q.y;
      }
    }
  }
}

// colv: this warp's [2][BN] shared-memory column vectors (bias, gate*alpha)
template <int BN, int EPI, bool SWAP>
__device__ __forceinline__ void epi_prefetch(const GemmDev& p, EpiPre& e,
                                             float* colv, int arow, int bcol0,
                                             int split, int lane) {
  const bool use_bias = p.bias != nullptr && (EPI != FVB_EPI_F32_ACC || split == 0);
  if (!SWAP) {
    const int n_feat = p.n;
    if (EPI == FVB_EPI_BF16 || EPI == FVB_EPI_F32_STORE || EPI == FVB_EPI_F32_ACC) {
      __syncwarp();  // the previous tile's readers are done
#pragma unroll 1
      for (int c = lane; c < BN; c += 32) {
        const int fc = min(bcol0 + c, n_feat - 1);
        colv[c] = use_bias ? __ldg(p.bias + fc) : 0.f;
        colv[BN + c] = (EPI == FVB_EPI_F32_ACC)
                           ? p.alpha * (p.gate ? __ldg(p.gate + fc) : 1.f) : 1.f;
      }
    }
    if (EPI == FVB_EPI_QKV_ROPE) {
      e.pos = arow < p.m ? p.positions[arow] : 0;
      const int qk_end = (p.n_heads + 1) * p.head_dim;
      if (bcol0 < qk_end) {
        float cs[32];
        load_rope32<BN, EPI>(p, e.pos, bcol0, cs);
#pragma unroll
        for (int j = 0; j < 16; ++j) { e.x0[j] = cs[j]; e.y0[j] = cs[16 + j]; }
      }
    }
  } else {
    const int n_feat = p.m;
    const int fs = min(arow, n_feat - 1);
    e.fb = use_bias ? __ldg(p.bias + fs) : 0.f;
    e.fg = p.alpha * (p.gate ? __ldg(p.gate + fs) : 1.f);
    const int hd = EPI == FVB_EPI_QKV_ROPE ? p.head_dim : 2;
    const bool is_qk = EPI == FVB_EPI_QKV_ROPE && arow < (p.n_heads + 1) * p.head_dim;
    swap_chunk_operands<EPI>(p, fs, is_qk, (arow % hd) >> 1, bcol0, e.x0, e.y0);
  }
}

// ---------------------------------------------------------------------------
// Normal orientation epilogue: thread = token row (t_base + lane), BN
// feature columns from bcol0, processed 32 at a time through the warp's
// staging block.  Vectorised write-back needs 16-byte aligned rows; other
// shapes use per-thread stores.
// ---------------------------------------------------------------------------
template <int BN, int EPI, int ACT>
__device__ __forceinline__ void epilogue_normal(const GemmDev& p, const EpiPre& e,
                                                const float* colv,
                                                uint32_t taddr, uint32_t* stage,
                                                int t_base, int bcol0, int lane) {
  const int n_tok = p.m, n_feat = p.n;
  const int t = t_base + lane;
  const bool row_ok = t < n_tok;
  const int rows_valid = min(32, n_tok - t_base);
  uint32_t* srow = stage + lane * STAGE_PITCH;
  const int hd = p.head_dim, half = hd >> 1;
  const int qk_end = (p.n_heads + 1) * hd;
  float cs[32];
  if (EPI == FVB_EPI_QKV_ROPE) {
#pragma unroll
    for (int j = 0; j < 16; ++j) { cs[j] = e.x0[j]; cs[16 + j] = e.y0[j]; }
  }
  __syncwarp();  // column vectors visible
#pragma unroll 1
  for (int g = 0; g < BN / 32; ++g) {
    const int c = g * 32;
    const int f0 = bcol0 + c;
    if (f0 >= n_feat) break;  // uniform across the warp
    const int ncol = min(32, n_feat - f0);
    uint32_t r0[16], r1[16];
    tmem_ld16_sync(taddr + (uint32_t)c, r0);
    tmem_ld16_sync(taddr + (uint32_t)(c + 16), r1);
    float v[32];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      v[j] = u2f(r0[j]);
      v[16 + j] = u2f(r1[j]);
    }
    // next group's rotary table, in flight while this group is processed
    float cs_next[32];
    if (EPI == FVB_EPI_QKV_ROPE && g + 1 < BN / 32 && f0 + 32 < qk_end)
      load_rope32<BN, EPI>(p, e.pos, f0 + 32, cs_next);

    if (EPI == FVB_EPI_BF16) {
      if (p.res || p.gate_tok) {
        // this row's residual / gate values of the 32 columns (n % 8 == 0)
        uint4 rq[4], gq[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const bool in = row_ok && f0 + 8 * q < n_feat;
          rq[q] = (in && p.res)
                      ? *reinterpret_cast<const uint4*>(p.res + (long long)t * p.ld_res + f0 + 8 * q)
                      : make_uint4(0u, 0u, 0u, 0u);
          gq[q] = (in && p.gate_tok)
                      ? *reinterpret_cast<const uint4*>(p.gate_tok + (long long)t * p.ld_gate_tok +
                                                        f0 + 8 * q)
                      : make_uint4(0x3f803f80u, 0x3f803f80u, 0x3f803f80u, 0x3f803f80u);
        }
        const bf16* rb = reinterpret_cast<const bf16*>(rq);
        const bf16* gb = reinterpret_cast<const bf16*>(gq);
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float y0 = apply_act<ACT>(p.alpha * v[j] + colv[c + j]) * __bfloat162float(gb[j]) +
                           __bfloat162float(rb[j]);
          const float y1 =
              apply_act<ACT>(p.alpha * v[j + 1] + colv[c + j + 1]) * __bfloat162float(gb[j + 1]) +
              __bfloat162float(rb[j + 1]);
          srow[j >> 1] = pack_bf16x2(y0, y1);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; j += 2)
          srow[j >> 1] = pack_bf16x2(apply_act<ACT>(p.alpha * v[j] + colv[c + j]),
                                     apply_act<ACT>(p.alpha * v[j + 1] + colv[c + j + 1]));
      }
      __syncwarp();
      bf16* base = reinterpret_cast<bf16*>(p.out) + (long long)t_base * p.ldo + f0;
      if ((p.ldo % 8) == 0 && (ncol % 8) == 0) {
        warp_writeback<16, 0>(stage, lane, rows_valid, ncol / 2, [&](int row) {
          return reinterpret_cast<uint32_t*>(base + (long long)row * p.ldo);
        });
      } else if (row_ok) {
        bf16* o = base + (long long)lane * p.ldo;
        for (int j = 0; j < ncol; ++j) {
          const uint32_t w = srow[j >> 1];
          o[j] = __ushort_as_bfloat16((j & 1) ? (unsigned short)(w >> 16)
                                              : (unsigned short)(w & 0xffff));
        }
      }
    } else if (EPI == FVB_EPI_F32_STORE || EPI == FVB_EPI_F32_ACC) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float y = (EPI == FVB_EPI_F32_STORE ? p.alpha * v[j] : v[j]) + colv[c + j];
        if (EPI == FVB_EPI_F32_ACC) y *= colv[BN + c + j];
        srow[j] = __float_as_uint(y);
      }
      __syncwarp();
      float* base = reinterpret_cast<float*>(p.out) + (long long)t_base * p.ldo + f0;
      auto dst = [&](int row) {
        return reinterpret_cast<uint32_t*>(base + (long long)row * p.ldo);
      };
      if ((p.ldo % 4) == 0) {
        if (EPI == FVB_EPI_F32_STORE) {
          if (p.row_add)
            warp_writeback<32, 3>(stage, lane, rows_valid, ncol, dst, 0,
                                  p.row_add + f0, p.row_add_mod, n_feat, t_base);
          else
            warp_writeback<32, 0>(stage, lane, rows_valid, ncol, dst);
        } else if (p.split > 1) {
          warp_writeback<32, 2>(stage, lane, rows_valid, ncol, dst);
        } else {
          warp_writeback<32, 1>(stage, lane, rows_valid, ncol, dst);
        }
      } else if (row_ok) {
        float* o = base + (long long)lane * p.ldo;
        for (int j = 0; j < ncol; ++j) {
          const float y = u2f(srow[j]);
          if (EPI == FVB_EPI_F32_STORE) {
            o[j] = p.row_add
                       ? y + __bfloat162float(
                                 p.row_add[(long long)(t % p.row_add_mod) * n_feat + f0 + j])
                       : y;
          } else if (p.split > 1) {
            atomicAdd(o + j, y);
          } else {
            o[j] += y;
          }
        }
      }
    } else if (EPI == FVB_EPI_GEGLU) {
#pragma unroll
      for (int i = 0; i < 16; i += 2)
        srow[i >> 1] = pack_bf16x2(gelu_tanh_f(v[2 * i]) * v[2 * i + 1],
                                   gelu_tanh_f(v[2 * i + 2]) * v[2 * i + 3]);
      __syncwarp();
      bf16* base = reinterpret_cast<bf16*>(p.out) + (long long)t_base * p.ldo + (f0 >> 1);
      if ((p.ldo % 8) == 0 && (ncol % 16) == 0) {
        warp_writeback<8, 0>(stage, lane, rows_valid, ncol / 4, [&](int row) {
          return reinterpret_cast<uint32_t*>(base + (long long)row * p.ldo);
        });
      } else if (row_ok) {
        bf16* o = base + (long long)lane * p.ldo;
        for (int i = 0; 2 * i + 1 < ncol; ++i) {
          const uint32_t w = srow[i >> 1];
          o[i] = __ushort_as_bfloat16((i & 1) ? (unsigned short)(w >> 16)
                                              : (unsigned short)(w & 0xffff));
        }
      }
    } else {  // FVB_EPI_QKV_ROPE: n_feat, head_dim multiples of 32
      if (f0 < qk_end && p.rope_interleaved) {
        // rotary pairs stay adjacent: packed column order is the output order
        const int hh = f0 / hd;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float cc = cs[2 * i], sn = cs[2 * i + 1];
          const float a0 = v[2 * i], b0 = v[2 * i + 1];
          srow[i] = pack_bf16x2(a0 * cc - b0 * sn, b0 * cc + a0 * sn);
        }
        __syncwarp();
        bf16* base;
        long long ld;
        if (hh < p.n_heads) {
          base = reinterpret_cast<bf16*>(p.out) + (long long)t_base * p.ldo + hh * hd + (f0 % hd);
          ld = p.ldo;
        } else {
          base = p.k_out + (long long)t_base * p.ld_kv + (f0 % hd);
          ld = p.ld_kv;
        }
        warp_writeback<16, 0>(stage, lane, rows_valid, 16, [&](int row) {
          return reinterpret_cast<uint32_t*>(base + (long long)row * ld);
        });
      } else if (f0 < qk_end) {
        const int hh = f0 / hd;
        const int i0 = (f0 % hd) >> 1;
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float c0 = cs[2 * i], s0 = cs[2 * i + 1];
          const float c1 = cs[2 * i + 2], s1 = cs[2 * i + 3];
          const float a0 = v[2 * i], b0 = v[2 * i + 1];
          const float a1 = v[2 * i + 2], b1 = v[2 * i + 3];
          srow[i >> 1] = pack_bf16x2(a0 * c0 - b0 * s0, a1 * c1 - b1 * s1);
          srow[8 + (i >> 1)] = pack_bf16x2(b0 * c0 + a0 * s0, b1 * c1 + a1 * s1);
        }
        __syncwarp();
        bf16* base;
        long long ld;
        if (hh < p.n_heads) {
          base = reinterpret_cast<bf16*>(p.out) + (long long)t_base * p.ldo + hh * hd + i0;
          ld = p.ldo;
        } else {
          base = p.k_out + (long long)t_base * p.ld_kv + i0;
          ld = p.ld_kv;
        }
        // words 0..7 -> dims i0..i0+15, words 8..15 -> dims i0+half..
        warp_writeback<16, 0>(stage, lane, rows_valid, 16,
                              [&](int row) {
                                return reinterpret_cast<uint32_t*>(base + (long long)row * ld);
                              },
                              half / 2 - 8);
      } else {
#pragma unroll
        for (int j = 0; j < 32; j += 2) srow[j >> 1] = pack_bf16x2(v[j], v[j + 1]);
        __syncwarp();
        bf16* base = p.v_out + (long long)t_base * p.ld_kv + (f0 - qk_end);
        warp_writeback<16, 0>(stage, lane, rows_valid, 16, [&](int row) {
          return reinterpret_cast<uint32_t*>(base + (long long)row * p.ld_kv);
        });
      }
      if (g + 1 < BN / 32) {
#pragma unroll
        for (int j = 0; j < 32; ++j) cs[j] = cs_next[j];
      }
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Normal orientation epilogue through TMA: per group of 32 accumulator
// columns the warp converts its 32 rows into swizzled 32-row boxes in its
// shared-memory buffer and one lane issues an asynchronous TMA store (BF16,
// F32_STORE, GEGLU) or TMA f32 reduce-add (F32_ACC: out += y, which also
// merges K splits in L2).  The warp's 4 KB buffer holds two 2 KB box slots,
// so a box is written while the previous one is still being read by the
// TMA unit, and the TMEM read of the next group is issued before the
// current group is converted: TMEM latency, conversion and stores overlap.
// Boxes (32 rows each): f32 16 columns (64 B rows), bf16 32 columns (64 B
// rows), GEGLU 16 bf16 columns (32 B rows); the swizzle span equals the row
// size.  Swizzle of byte offset o inside a slot: the 16-byte chunk bits
// [4, 4+b) are XORed with bits [7, 7+b), b = log2(row bytes / 16).
// ---------------------------------------------------------------------------
template <int EPI>
struct TmaBox {
  static constexpr bool F32 = EPI == FVB_EPI_F32_STORE || EPI == FVB_EPI_F32_ACC;
  static constexpr int ROW_BYTES = EPI == FVB_EPI_GEGLU ? 32 : 64;
  static constexpr int COLS = F32 ? 16 : (EPI == FVB_EPI_GEGLU ? 16 : 32);
  static constexpr int PER_GROUP = F32 ? 2 : 1;  // boxes per 32 accumulator columns
  static constexpr uint32_t SW = ROW_BYTES == 64 ? 3u : 1u;
  static constexpr uint32_t SLOT = 2048;
};

template <int BN, int EPI, int ACT>
__device__ __forceinline__ void epilogue_tma(const GemmDev& p,
                                             const CUtensorMap* tmO,
                                             const float* colv, uint32_t taddr,
                                             uint8_t* buf, int t_base,
                                             int bcol0, int lane) {
  using BX = TmaBox<EPI>;
  constexpr int RB = BX::ROW_BYTES;
  constexpr int NCH = RB / 16;   // 16-byte chunks per box row
  constexpr int WPB = RB / 4;    // 32-bit words per box row
  if (t_base >= p.m) return;  // whole warp past the last token row
  const int ng = min(BN / 32, (p.n - bcol0 + 31) / 32);
  const uint32_t sbuf = smem_u32(buf);
  const uint32_t o_row = (uint32_t)(lane * RB);
  uint32_t slot = 0;
  uint32_t cur[32], nxt[32];
  tmem_ld32(taddr, cur);
  tmem_wait_ld32(cur);
  __syncwarp();  // column vectors visible
  const bool tr = p.trace && lane == 0 && (t_base & 127) == 64;
  if (tr) trace_stamp(p, 8);
#pragma unroll 1
  for (int g = 0; g < ng; ++g) {
    const int c = g * 32;
    if (g + 1 < ng) tmem_ld32(taddr + (uint32_t)(c + 32), nxt);
    uint32_t w[32];
    if (EPI == FVB_EPI_BF16) {
#pragma unroll
      for (int j = 0; j < 32; j += 2)
        w[j >> 1] = pack_bf16x2(
            apply_act<ACT>(p.alpha * u2f(cur[j]) + colv[c + j]),
            apply_act<ACT>(p.alpha * u2f(cur[j + 1]) + colv[c + j + 1]));
    } else if (EPI == FVB_EPI_GEGLU) {
#pragma unroll
      for (int i = 0; i < 16; i += 2)
        w[i >> 1] = pack_bf16x2(gelu_tanh_f(u2f(cur[2 * i])) * u2f(cur[2 * i + 1]),
                                gelu_tanh_f(u2f(cur[2 * i + 2])) * u2f(cur[2 * i + 3]));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float y = (EPI == FVB_EPI_F32_STORE ? p.alpha * u2f(cur[j]) : u2f(cur[j])) +
                  colv[c + j];
        if (EPI == FVB_EPI_F32_ACC) y *= colv[BN + c + j];
        w[j] = __float_as_uint(y);
      }
    }
#pragma unroll
    for (int bx = 0; bx < BX::PER_GROUP; ++bx) {
      if (lane == 0) bulk_wait_read1();  // this slot's previous box was read
      __syncwarp();
      const uint32_t sb = sbuf + slot * BX::SLOT;
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        const uint32_t o = o_row + (uint32_t)(ch * 16);
        const uint32_t phys = o ^ (((o >> 7) & BX::SW) << 4);
        const int w0 = bx * WPB + 4 * ch;
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sb + phys),
                     "r"(w[w0]), "r"(w[w0 + 1]), "r"(w[w0 + 2]), "r"(w[w0 + 3])
                     : "memory");
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int col = bcol0 + c + bx * BX::COLS;
        const int x = EPI == FVB_EPI_GEGLU ? col >> 1 : col;
        if (EPI == FVB_EPI_F32_ACC)
          tma_reduce_add_2d(tmO, x, t_base, buf + slot * BX::SLOT);
        else
          tma_store_2d(tmO, x, t_base, buf + slot * BX::SLOT);
        bulk_commit();
      }
      slot ^= 1u;
    }
    if (tr && g < 2) trace_stamp(p, 9 + g);
    if (g + 1 < ng) {
      tmem_wait_ld32(nxt);
#pragma unroll
      for (int j = 0; j < 32; ++j) cur[j] = nxt[j];
    }
  }
}

// ---------------------------------------------------------------------------
// Swapped orientation epilogue: thread = feature row f, BN token columns in
// chunks of 16, the next chunk's gathered operands loaded one chunk ahead.
// Consecutive lanes hold consecutive features, so per-token stores coalesce.
// ---------------------------------------------------------------------------
template <int BN, int EPI, int ACT, bool FROM_WS>
__device__ __forceinline__ void epilogue_swap(const GemmDev& p, const EpiPre& e,
                                              uint32_t taddr, const float* wst,
                                              int f, int bcol0, int lane) {
  const int n_tok = p.n, n_feat = p.m;
  const bool f_ok = f < n_feat;
  const int fs = min(f, n_feat - 1);
  const int hd = EPI == FVB_EPI_QKV_ROPE ? p.head_dim : 2;
  const int qk_end = (p.n_heads + 1) * p.head_dim;
  const bool is_qk = EPI == FVB_EPI_QKV_ROPE && f < qk_end;
  const int pair_i = (f % hd) >> 1;
  const bool second = (f % hd) & 1;
  float x[16], y[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) { x[j] = e.x0[j]; y[j] = e.y0[j]; }
#pragma unroll 1
  for (int c = 0; c < BN; c += 16) {
    const int t0 = bcol0 + c;
    if (t0 >= n_tok) break;  // uniform across the warp
    uint32_t r[16];
    if (FROM_WS) {
      const int fr = f & (GEMM_BM - 1);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        r[j] = __float_as_uint(__ldcg(wst + (c + j) * GEMM_BM + fr));
    } else {
      tmem_ld16_sync(taddr + (uint32_t)c, r);
    }
    float xn[16], yn[16];
    const bool more = c + 16 < BN && t0 + 16 < n_tok;
    if (more) swap_chunk_operands<EPI>(p, fs, is_qk, pair_i, t0 + 16, xn, yn);
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = u2f(r[j]);
    float other[16];
    if (EPI == FVB_EPI_GEGLU || EPI == FVB_EPI_QKV_ROPE) {
#pragma unroll
      for (int j = 0; j < 16; ++j) other[j] = __shfl_xor_sync(0xffffffffu, v[j], 1);
    }
    if (f_ok) {
      const int nj = min(16, n_tok - t0);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (j < nj) {
          const long long tt = t0 + j;
          if (EPI == FVB_EPI_BF16) {
            reinterpret_cast<bf16*>(p.out)[tt * p.ldo + f] =
                __float2bfloat16(apply_act<ACT>(p.alpha * v[j] + e.fb));
          } else if (EPI == FVB_EPI_F32_STORE) {
            reinterpret_cast<float*>(p.out)[tt * p.ldo + f] = p.alpha * (v[j] + x[j]) + e.fb;
          } else if (EPI == FVB_EPI_F32_ACC) {
            float* o = reinterpret_cast<float*>(p.out) + tt * p.ldo + f;
            if (p.split > 1)
              atomicAdd(o, (v[j] + e.fb) * e.fg);
            else
              *o = x[j] + (v[j] + e.fb) * e.fg;
          } else if (EPI == FVB_EPI_GEGLU) {
            if (!(lane & 1))
              reinterpret_cast<bf16*>(p.out)[tt * p.ldo + (f >> 1)] =
                  __float2bfloat16(gelu_tanh_f(v[j]) * other[j]);
          } else if (is_qk) {
            const int hh = f / hd;
            const float x1 = second ? other[j] : v[j];
            const float x2 = second ? v[j] : other[j];
            const float rr = second ? (x2 * x[j] + x1 * y[j]) : (x1 * x[j] - x2 * y[j]);
            const int dim = second ? pair_i + (hd >> 1) : pair_i;
            if (hh < p.n_heads)
              reinterpret_cast<bf16*>(p.out)[tt * p.ldo + hh * hd + dim] = __float2bfloat16(rr);
            else
              p.k_out[tt * p.ld_kv + dim] = __float2bfloat16(rr);
          } else {
            p.v_out[tt * p.ld_kv + (f - qk_end)] = __float2bfloat16(v[j]);
          }
        }
      }
    }
    if (more) {
#pragma unroll
      for (int j = 0; j < 16; ++j) { x[j] = xn[j]; y[j] = yn[j]; }
    }
  }
}

template <int BN, int STAGES, int EPI, bool SWAP, int ACT>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO, const GemmDev p) {
  constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  constexpr int B_BYTES = BN * GEMM_BK * 2;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t IDESC = idesc_bf16_f32(GEMM_BM, BN);
  // two accumulators; the allocation is a power of two >= 32 columns
  constexpr uint32_t TMEM_COLS = 2 * BN <= 128 ? 2 * BN : (2 * BN <= 256 ? 256 : 512);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // [ring][epilogue staging (1024-aligned; per-warp 4 KB TMA boxes or
  // 32 x 33-word staging blocks)][column vectors][barriers]
  uint32_t* stage_all = reinterpret_cast<uint32_t*>(smem + STAGES * STAGE_BYTES);
  float* colv_all = reinterpret_cast<float*>(stage_all + 4 * 32 * STAGE_PITCH);  // [4][2][BN]
  uint64_t* full = reinterpret_cast<uint64_t*>(colv_all + 4 * 2 * BN);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;   // [2]
  uint64_t* tempty = tfull + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* fix_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    trace_stamp(p, 0);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    fence_barrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    if (p.tma_out) prefetch_tensormap(&tmO);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) trace_stamp(p, 1);

  if (warp == 0) {
    if (lane == 0) {
      // the weights are the A operand in the swapped orientation
      const CUtensorMap* mw = SWAP ? &tmA : &tmB;
      const CUtensorMap* mx = SWAP ? &tmB : &tmA;
      constexpr int woff = SWAP ? 0 : A_BYTES;
      constexpr int xoff = SWAP ? A_BYTES : 0;
      int it = 0;
      bool alive = true;
      bool waited = false;
      for (int w = blockIdx.x; w < p.n_work && alive; w += gridDim.x) {
        const Tile t = decode_tile(p, w);
        const int n0 = t.nt * BN;
        const int wrow = SWAP ? t.m0 : n0, xrow = SWAP ? n0 : t.m0;
        int kt = t.kt0;
        if (!waited) {
          // first tile: stream the weights of the first stages before
          // waiting for the kernel that produces the activations
          const int npre = min(STAGES, t.kt1 - t.kt0);
          for (int i = 0; i < npre; ++i) {
            mbar_arrive_expect_tx(&full[i], STAGE_BYTES);
            tma_load_2d(smem + i * STAGE_BYTES + woff, mw,
                        (t.kt0 + i) * GEMM_BK, wrow, &full[i]);
          }
          trace_stamp(p, 2);
          griddep_wait();
          waited = true;
          for (int i = 0; i < npre; ++i)
            tma_load_2d(smem + i * STAGE_BYTES + xoff, mx,
                        (t.kt0 + i) * GEMM_BK, xrow, &full[i]);
          it = npre;
          kt += npre;
        }
        for (; kt < t.kt1; ++kt, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1)) { alive = false; break; }
          uint8_t* sa = smem + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          tma_load_2d(sa + woff, mw, kt * GEMM_BK, wrow, &full[s]);
          tma_load_2d(sa + xoff, mx, kt * GEMM_BK, xrow, &full[s]);
        }
      }
      if (!waited) griddep_wait();
      griddep_launch_dependents();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, j = 0;
      bool alive = true;
      for (int w = blockIdx.x; w < p.n_work && alive; w += gridDim.x, ++j) {
        const Tile t = decode_tile(p, w);
        const int acc = j & 1;
        if (!mbar_wait(&tempty[acc], ((j >> 1) & 1) ^ 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(acc * BN);
        for (int kt = t.kt0; kt < t.kt1; ++kt, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph)) { alive = false; break; }
          tc_fence_after();
          if (it == 0) trace_stamp(p, 3);
          const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
          const uint64_t da = smem_desc_sw128(sa);
          const uint64_t db = smem_desc_sw128(sa + A_BYTES);
#pragma unroll
          for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
            // +32 bytes per K=16 step inside the 128-byte swizzled row
            tc_mma_bf16(d_tmem, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2),
                        IDESC, (kt > t.kt0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (alive) tc_commit(&tfull[acc]);
      }
      trace_stamp(p, 4);
    }
  } else {
    const int q = warp & 3;
    uint32_t* stage = stage_all + q * 32 * STAGE_PITCH;
    float* colv = colv_all + q * 2 * BN;
    griddep_wait();
    int j = 0;
    for (int w = blockIdx.x; w < p.n_work; w += gridDim.x, ++j) {
      const Tile t = decode_tile(p, w);
      const int acc = j & 1;
      EpiPre pre;
      epi_prefetch<BN, EPI, SWAP>(p, pre, colv, t.m0 + q * 32 + lane,
                                  t.nt * BN, t.split, lane);
      const bool ok = mbar_wait(&tfull[acc], (j >> 1) & 1);
      __syncwarp();
      if (!ok) break;
      tc_fence_after();
      if (j == 0 && warp == 2 && lane == 0) trace_stamp(p, 5);
      const uint32_t taddr =
          tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      if (SWAP && EPI != FVB_EPI_F32_ACC && p.split > 1) {
        // split-K: add this split's partial into the tile workspace ...
        const int tile_mn = w % (p.m_tiles * p.n_tiles);
        float* wst = p.ws + (long long)tile_mn * BN * GEMM_BM;
        const int fr = q * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          uint32_t r[16];
          tmem_ld16_sync(taddr + (uint32_t)c, r);
#pragma unroll
          for (int jj = 0; jj < 16; ++jj)
            atomicAdd(wst + (c + jj) * GEMM_BM + fr, u2f(r[jj]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        // ... and the last split to arrive runs the epilogue on the sum
        __threadfence();
        epi_bar_sync();
        if (warp == 2 && lane == 0)
          *fix_flag = (atomicAdd(p.ws_cnt + tile_mn, 1u) == (unsigned)(p.split - 1));
        epi_bar_sync();
        if (*fix_flag) {
          __threadfence();
          epilogue_swap<BN, EPI, ACT, true>(p, pre, 0, wst, t.m0 + fr,
                                            t.nt * BN, lane);
#pragma unroll 4
          for (int c = 0; c < BN; ++c) wst[c * GEMM_BM + fr] = 0.f;
          if (warp == 2 && lane == 0) p.ws_cnt[tile_mn] = 0u;
        }
        continue;
      }
      if (SWAP)
        epilogue_swap<BN, EPI, ACT, false>(p, pre, taddr, nullptr,
                                           t.m0 + q * 32 + lane, t.nt * BN,
                                           lane);
      else if (EPI != FVB_EPI_QKV_ROPE && p.tma_out)
        epilogue_tma<BN, EPI, ACT>(p, &tmO, colv, taddr,
                                   reinterpret_cast<uint8_t*>(stage_all) + q * 4096,
                                   t.m0 + q * 32, t.nt * BN, lane);
      else
        epilogue_normal<BN, EPI, ACT>(p, pre, colv, taddr, stage, t.m0 + q * 32,
                                      t.nt * BN, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (warp == 2 && lane == 0) trace_stamp(p, 11);
    if (!SWAP && lane == 0) bulk_wait0();  // TMA stores complete before exit
    if (warp == 2 && lane == 0) trace_stamp(p, 12);
    if (warp == 2 && lane == 0) trace_stamp(p, 6);
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace_stamp(p, 7);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (!SWAP && p.norm_out) {
    // every CTA's output tiles are complete (TMA reductions waited above),
    // then the CTAs normalise the finished rows, one warp per row
    __threadfence();
    __syncthreads();
    volatile int* go = reinterpret_cast<volatile int*>(fix_flag);
    if (threadIdx.x == 0) {
      const unsigned long long add =
          blockIdx.x == 0 ? NORM_SYNC_UNIT - gridDim.x + 1 : 1ull;
      unsigned long long old;
      asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], %2;"
                   : "=l"(old) : "l"(p.norm_sync), "l"(add) : "memory");
      const unsigned long long target = (old / NORM_SYNC_UNIT + 1) * NORM_SYNC_UNIT;
      bool ok = true;
      const uint64_t t0 = globaltimer_ns();
      for (unsigned n = 0;; ++n) {
        unsigned long long v;
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p.norm_sync) : "memory");
        if (v >= target) break;
        if ((n & 255) == 255 && globaltimer_ns() - t0 > FVB_WAIT_LIMIT_NS) {
          record_device_error(FVB_ERR_DEVICE_TIMEOUT);
          ok = false;
          break;
        }
      }
      *go = ok;
    }
    __syncthreads();
    if (*go) {
      constexpr int NW = GEMM_THREADS / 32;
      for (int row = blockIdx.x * NW + warp; row < p.m; row += gridDim.x * NW)
        norm_row_warp(p.norm_mode, reinterpret_cast<const float*>(p.out) + (long long)row * p.ldo,
                      p.norm_out + (long long)row * p.ld_norm_out, p.n, p.norm_w,
                      p.norm_b, p.norm_eps, lane);
    }
  }
}

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = (BN == 64) ? 8 : (BN == 128 ? 6 : (BN == 192 ? 5 : 4));
  static_assert(BN % 32 == 0 && BN <= 256, "block_n");
  static constexpr int SMEM = STAGES * (GEMM_BM * GEMM_BK * 2 + BN * GEMM_BK * 2) +
                              1024 + 4 * 32 * STAGE_PITCH * 4 + 4 * 2 * BN * 4 + 256;
};

}  // namespace fvb
