// tcgen05 / TMEM tensor-core GEMM for sm_100a:  C[M,N] = A[M,K] * B[N,K]^T.
//
// One CTA computes one 128 x BN output tile:
//   warp 0 (one lane)  : TMA producer, STAGES-deep ring of (A,B) k-tiles
//                        (64 bf16 = 128 B per row, 128-byte swizzle)
//   warp 1             : allocates BN TMEM columns; one lane issues
//                        tcgen05.mma (M=128, N=BN, K=16) x4 per k-tile and
//                        commits each stage back to the producer
//   warps 2..5         : epilogue; warp w reads TMEM lanes 32*(w%4)..+31
//                        (one accumulator row per thread) with tcgen05.ld
//                        and applies the fused epilogue.
// The epilogue works on (token, feature) pairs: in the normal orientation A
// rows are tokens and B rows are features; with `swap` A rows are features
// (the weight matrix streams through the M side) and B rows are tokens, which
// is how the denoise loop runs its 50/51-token GEMMs on tensor cores.
#pragma once

#include "common.cuh"

namespace fvb {

struct GemmDev {
  int m, n, k;
  int swap, epi, act;
  int k_tiles, kt_per_split, split;
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
};

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_THREADS = 192;

__device__ __forceinline__ float apply_act(float x, int act) {
  if (act == FVB_ACT_GELU_TANH) return gelu_tanh_f(x);
  if (act == FVB_ACT_SILU) return silu_f(x);
  return x;
}

// Epilogue for 16 accumulator values of one A row (`arow`, absolute) and B
// rows bcol0 .. bcol0+15 (absolute).  All 32 lanes of the warp call this
// together (shuffles in the swapped orientation).
__device__ __forceinline__ void gemm_epilogue16(const GemmDev& p, int arow,
                                                int bcol0, float (&v)[16],
                                                int lane) {
  const bool swap = p.swap != 0;
  const int n_tok = swap ? p.n : p.m;
  const int n_feat = swap ? p.m : p.n;

  if (p.epi == FVB_EPI_GEGLU || p.epi == FVB_EPI_QKV_ROPE) {
    // Paired features: packed feature 2i and 2i+1 belong together.
    float other[16];
    if (swap) {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        other[j] = __shfl_xor_sync(0xffffffffu, v[j], 1);
    }
    if (p.epi == FVB_EPI_GEGLU) {
      bf16* out = reinterpret_cast<bf16*>(p.out);
      if (!swap) {
        const int t = arow;
        if (t >= n_tok) return;
        const int f0 = bcol0 >> 1;
        if (bcol0 + 16 <= n_feat) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            w[i] = pack_bf16x2(gelu_tanh_f(v[4 * i]) * v[4 * i + 1],
                               gelu_tanh_f(v[4 * i + 2]) * v[4 * i + 3]);
          *reinterpret_cast<uint4*>(out + (long long)t * p.ldo + f0) =
              make_uint4(w[0], w[1], w[2], w[3]);
        } else {
          for (int i = 0; i < 8; ++i)
            if (bcol0 + 2 * i + 1 < n_feat)
              out[(long long)t * p.ldo + f0 + i] =
                  __float2bfloat16(gelu_tanh_f(v[2 * i]) * v[2 * i + 1]);
        }
      } else {
        const int f = arow;
        if ((lane & 1) || f >= n_feat) return;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int t = bcol0 + j;
          if (t < n_tok)
            out[(long long)t * p.ldo + (f >> 1)] =
                __float2bfloat16(gelu_tanh_f(v[j]) * other[j]);
        }
      }
      return;
    }
    // QKV + RoPE
    const int hd = p.head_dim, half = hd >> 1;
    const int qk_end = (p.n_heads + 1) * hd;
    bf16* qout = reinterpret_cast<bf16*>(p.out);
    if (!swap) {
      const int t = arow;
      if (t >= n_tok || bcol0 >= n_feat) return;
      if (bcol0 < qk_end) {
        const int hh = bcol0 / hd;
        const int i0 = (bcol0 % hd) >> 1;  // 8 consecutive dims i0..i0+7
        const int pos = p.positions[t];
        const float* cs = p.rope_cs + ((long long)pos * half + i0) * 2;
        float o1[8], o2[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float c = cs[2 * i], s = cs[2 * i + 1];
          const float x1 = v[2 * i], x2 = v[2 * i + 1];
          o1[i] = x1 * c - x2 * s;
          o2[i] = x2 * c + x1 * s;
        }
        bf16* dst = (hh < p.n_heads)
                        ? qout + (long long)t * p.ldo + hh * hd
                        : p.k_out + (long long)t * p.ld_kv;
        uint4 a = make_uint4(pack_bf16x2(o1[0], o1[1]), pack_bf16x2(o1[2], o1[3]),
                             pack_bf16x2(o1[4], o1[5]), pack_bf16x2(o1[6], o1[7]));
        uint4 b = make_uint4(pack_bf16x2(o2[0], o2[1]), pack_bf16x2(o2[2], o2[3]),
                             pack_bf16x2(o2[4], o2[5]), pack_bf16x2(o2[6], o2[7]));
        *reinterpret_cast<uint4*>(dst + i0) = a;
        *reinterpret_cast<uint4*>(dst + i0 + half) = b;
      } else {
        const int d0 = bcol0 - qk_end;
        bf16* dst = p.v_out + (long long)t * p.ld_kv + d0;
        uint4 a = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                             pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
        uint4 b = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]),
                             pack_bf16x2(v[12], v[13]), pack_bf16x2(v[14], v[15]));
        *reinterpret_cast<uint4*>(dst) = a;
        *reinterpret_cast<uint4*>(dst + 8) = b;
      }
    } else {
      const int f = arow;
      if (f >= n_feat) return;
      if (f < qk_end) {
        const int hh = f / hd;
        const int within = f % hd;
        const int i = within >> 1;
        const bool second = within & 1;
        bf16* dst = (hh < p.n_heads) ? qout + hh * hd : p.k_out;
        const long long ld = (hh < p.n_heads) ? p.ldo : p.ld_kv;
        const int dim = second ? i + half : i;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int t = bcol0 + j;
          if (t >= n_tok) break;
          const int pos = p.positions[t];
          const float c = p.rope_cs[((long long)pos * half + i) * 2];
          const float s = p.rope_cs[((long long)pos * half + i) * 2 + 1];
          const float x1 = second ? other[j] : v[j];
          const float x2 = second ? v[j] : other[j];
          const float r = second ? (x2 * c + x1 * s) : (x1 * c - x2 * s);
          dst[(long long)t * ld + dim] = __float2bfloat16(r);
        }
      } else {
        const int d = f - qk_end;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int t = bcol0 + j;
          if (t >= n_tok) break;
          p.v_out[(long long)t * p.ld_kv + d] = __float2bfloat16(v[j]);
        }
      }
    }
    return;
  }

  // Unpaired epilogues: element (t, f).
  const bool use_bias = p.bias != nullptr && (p.epi != FVB_EPI_F32_ACC ||
                                              blockIdx.z == 0);
  if (!swap) {
    const int t = arow;
    if (t >= n_tok) return;
    const bool full = (bcol0 + 16 <= n_feat);
    if (p.epi == FVB_EPI_BF16) {
      bf16* out = reinterpret_cast<bf16*>(p.out) + (long long)t * p.ldo;
      float y[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int f = bcol0 + j;
        const float b = (use_bias && f < n_feat) ? p.bias[f] : 0.f;
        y[j] = apply_act(p.alpha * v[j] + b, p.act);
      }
      if (full && (p.ldo % 8) == 0) {
        uint4 a = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                             pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
        uint4 b = make_uint4(pack_bf16x2(y[8], y[9]), pack_bf16x2(y[10], y[11]),
                             pack_bf16x2(y[12], y[13]), pack_bf16x2(y[14], y[15]));
        *reinterpret_cast<uint4*>(out + bcol0) = a;
        *reinterpret_cast<uint4*>(out + bcol0 + 8) = b;
      } else {
        for (int j = 0; j < 16; ++j)
          if (bcol0 + j < n_feat) out[bcol0 + j] = __float2bfloat16(y[j]);
      }
    } else if (p.epi == FVB_EPI_F32_STORE) {
      float* out = reinterpret_cast<float*>(p.out) + (long long)t * p.ldo;
      const bf16* ra = p.row_add ? p.row_add + (long long)(t % p.row_add_mod) *
                                                   n_feat
                                 : nullptr;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int f = bcol0 + j;
        if (f < n_feat) {
          float y = v[j];
          if (use_bias) y += p.bias[f];
          if (ra) y += __bfloat162float(ra[f]);
          out[f] = y;
        }
      }
    } else {  // FVB_EPI_F32_ACC
      float* out = reinterpret_cast<float*>(p.out) + (long long)t * p.ldo;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int f = bcol0 + j;
        if (f < n_feat) {
          float y = v[j];
          if (use_bias) y += p.bias[f];
          y *= p.alpha;
          if (p.gate) y *= p.gate[f];
          if (p.split > 1)
            atomicAdd(out + f, y);
          else
            out[f] += y;
        }
      }
    }
  } else {
    const int f = arow;
    if (f >= n_feat) return;
    const float b = use_bias ? p.bias[f] : 0.f;
    if (p.epi == FVB_EPI_BF16) {
      bf16* out = reinterpret_cast<bf16*>(p.out) + f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int t = bcol0 + j;
        if (t < n_tok)
          out[(long long)t * p.ldo] =
              __float2bfloat16(apply_act(p.alpha * v[j] + b, p.act));
      }
    } else if (p.epi == FVB_EPI_F32_STORE) {
      float* out = reinterpret_cast<float*>(p.out) + f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int t = bcol0 + j;
        if (t < n_tok) {
          float y = v[j] + b;
          if (p.row_add)
            y += __bfloat162float(
                p.row_add[(long long)(t % p.row_add_mod) * n_feat + f]);
          out[(long long)t * p.ldo] = y;
        }
      }
    } else {
      float* out = reinterpret_cast<float*>(p.out) + f;
      const float g = p.alpha * (p.gate ? p.gate[f] : 1.f);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int t = bcol0 + j;
        if (t < n_tok) {
          const float y = (v[j] + b) * g;
          if (p.split > 1)
            atomicAdd(out + (long long)t * p.ldo, y);
          else
            out[(long long)t * p.ldo] += y;
        }
      }
    }
  }
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB, const GemmDev p) {
  constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  constexpr int B_BYTES = BN * GEMM_BK * 2;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t IDESC = idesc_bf16_f32(GEMM_BM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * GEMM_BM, n0 = blockIdx.y * BN;
  const int kt0 = blockIdx.z * p.kt_per_split;
  const int kt1 = min(kt0 + p.kt_per_split, p.k_tiles);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    fence_barrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (kt1 > kt0) {
    if (warp == 0) {
      if (lane == 0) {
        int it = 0;
        for (int kt = kt0; kt < kt1; ++kt, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1)) break;
          uint8_t* sa = smem + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          tma_load_2d(sa, &tmA, kt * GEMM_BK, m0, &full[s]);
          tma_load_2d(sa + A_BYTES, &tmB, kt * GEMM_BK, n0, &full[s]);
        }
      }
    } else if (warp == 1) {
      if (lane == 0) {
        int it = 0;
        bool ok = true;
        for (int kt = kt0; kt < kt1; ++kt, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
          const uint64_t da = smem_desc_sw128(sa);
          const uint64_t db = smem_desc_sw128(sa + A_BYTES);
#pragma unroll
          for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
            // +32 bytes per K=16 step inside the 128-byte swizzled row
            tc_mma_bf16(tmem, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2),
                        IDESC, (kt > kt0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (ok) tc_commit(tfull);
      }
    } else {
      const int q = warp & 3;
      const bool ok = mbar_wait(tfull, 0);
      __syncwarp();
      if (ok) {
        tc_fence_after();
        const int arow = m0 + q * 32 + lane;
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          float v[16];
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
          gemm_epilogue16(p, arow, n0 + c, v, lane);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = (BN == 64) ? 8 : (BN == 128 ? 6 : 4);
  static constexpr int SMEM =
      STAGES * (GEMM_BM * GEMM_BK * 2 + BN * GEMM_BK * 2) + 1024 + 256;
};

}  // namespace fvb
