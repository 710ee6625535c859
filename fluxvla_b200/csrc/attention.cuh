// Fused masked attention (flash-style online softmax, nothing of the
// [queries x keys] logits matrix goes to HBM).
//
// CTA = 64 query rows of one (batch, head) x one range of keys; 4 warps, 16
// rows each, bf16 mma.sync m16n8k16 with f32 accumulation; K/V tiles of 64
// keys double-buffered in shared memory with cp.async.  head_dim 256 (Gemma,
// MQA with 8 query heads on 1 KV head) and 72 (SigLIP, padded to 80 with
// zero columns) are instantiated.  With kv_splits > 1 each CTA writes an
// un-normalised partial (O, m, l) to the workspace and
// attn_combine_kernel merges the splits (the denoise loop has only 51
// queries per head, so it splits over the ~870 keys to use the whole GPU).
#pragma once

#include "common.cuh"

namespace fvb {

struct AttnDev {
  const bf16* q;
  long long q_rs, q_hs;
  const bf16* k;
  long long k_rs, k_hs;
  const bf16* v;
  long long v_rs, v_hs;
  bf16* o;
  long long o_rs, o_hs;
  int n_q, n_kv, heads, group, batch;
  long long q_br, kv_br;
  float scale_log2;  // scale * log2(e)
  const uint8_t* key_valid;
  int n_prefix;
  const int* q_block;
  const int* k_block;
  int splits, blocks_per_split;
  float* part_o;   // [splits][batch*heads][n_q][HD]
  float* part_ml;  // [splits][batch*heads][n_q][2]
};

constexpr int ATT_BM = 64, ATT_BN = 64, ATT_THREADS = 128;

__device__ __forceinline__ void cp_async16(void* sdst, const void* gsrc,
                                           bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                   smem_u32(sdst)),
               "l"(gsrc), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0,
                                        uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0,
                                          uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0,
                                               uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Load `rows` rows of HD bf16 (row stride rs elements) into a smem tile with
// row pitch PITCH elements; rows >= valid_rows are zero-filled.
template <int HD, int PITCH>
__device__ __forceinline__ void load_tile_async(bf16* s, const bf16* g,
                                                long long rs, int valid_rows,
                                                int tid) {
  constexpr int CH = HD * 2 / 16;  // 16-byte chunks per row
  for (int c = tid; c < 64 * CH; c += ATT_THREADS) {
    const int r = c / CH, cc = c % CH;
    const bool ok = r < valid_rows;
    const bf16* src = ok ? g + (long long)r * rs + cc * 8 : g;
    cp_async16(s + r * PITCH + cc * 8, src, ok);
  }
}

template <int HD, int HDP>
__global__ void __launch_bounds__(ATT_THREADS)
    attn_kernel(const AttnDev p) {
  constexpr int PITCH = HDP + 8;
  constexpr int TILE = 64 * PITCH;
  constexpr int NT_D = HDP / 8;  // output n-tiles
  extern __shared__ __align__(16) uint8_t smem_raw[];
  bf16* sQ = reinterpret_cast<bf16*>(smem_raw);
  bf16* sK = sQ + TILE;      // [2][TILE]
  bf16* sV = sK + 2 * TILE;  // [2][TILE]
  uint8_t* sMask = reinterpret_cast<uint8_t*>(sV + 2 * TILE);  // [2][64]
  int* sKb = reinterpret_cast<int*>(sMask + 128);              // [2][64]

  griddep_wait();
  griddep_launch_dependents();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = blockIdx.x * ATT_BM;
  const int h = blockIdx.y;
  const int bz = blockIdx.z;
  const int b = bz / p.splits, split = bz % p.splits;
  const int kvh = h / p.group;
  const int nkb = (p.n_kv + ATT_BN - 1) / ATT_BN;
  const int kb0 = split * p.blocks_per_split;
  const int kb1 = min(kb0 + p.blocks_per_split, nkb);

  const bf16* gq = p.q + ((long long)b * p.q_br + q0) * p.q_rs + h * p.q_hs;
  const bf16* gk = p.k + (long long)b * p.kv_br * p.k_rs + kvh * p.k_hs;
  const bf16* gv = p.v + (long long)b * p.kv_br * p.v_rs + kvh * p.v_hs;

  // zero the padding columns HD..HDP-1 (never written by cp.async)
  if (HDP > HD) {
    for (int r = tid; r < 5 * 64; r += ATT_THREADS)
      for (int c = HD; c < HDP; ++c) sQ[r * PITCH + c] = __float2bfloat16(0.f);
  }

  auto load_kv = [&](int kb, int buf) {
    const int k0 = kb * ATT_BN;
    const int nv = min(ATT_BN, p.n_kv - k0);
    load_tile_async<HD, PITCH>(sK + buf * TILE, gk + (long long)k0 * p.k_rs,
                               p.k_rs, nv, tid);
    load_tile_async<HD, PITCH>(sV + buf * TILE, gv + (long long)k0 * p.v_rs,
                               p.v_rs, nv, tid);
    if (tid < ATT_BN) {
      const int j = k0 + tid;
      uint8_t vis = j < p.n_kv;
      int kbv = 0;
      if (vis) {
        if (j < p.n_prefix) {
          vis = p.key_valid ? (p.key_valid[j] != 0) : 1;
        } else if (p.k_block) {
          kbv = p.k_block[j - p.n_prefix];
        }
      }
      sMask[buf * 64 + tid] = vis;
      sKb[buf * 64 + tid] = kbv;
    }
  };

  load_tile_async<HD, PITCH>(sQ, gq, p.q_rs, min(ATT_BM, p.n_q - q0), tid);
  if (kb0 < kb1) load_kv(kb0, 0);
  cp_async_commit();

  // query rows of this thread (within the tile): r0 = lane/4, r1 = r0 + 8
  const int qr0 = q0 + warp * 16 + (lane >> 2);
  const int qr1 = qr0 + 8;
  const int qb0 = (p.q_block && qr0 < p.n_q) ? p.q_block[qr0] : 0x7fffffff;
  const int qb1 = (p.q_block && qr1 < p.n_q) ? p.q_block[qr1] : 0x7fffffff;

  float o[NT_D][4];
#pragma unroll
  for (int i = 0; i < NT_D; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  const uint32_t sQa = smem_u32(sQ);
  for (int kb = kb0; kb < kb1; ++kb) {
    const int buf = (kb - kb0) & 1;
    if (kb + 1 < kb1) {
      load_kv(kb + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();

    const uint32_t sKa = smem_u32(sK + buf * TILE);
    const uint32_t sVa = smem_u32(sV + buf * TILE);
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HDP / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      {
        const int row = warp * 16 + (lane & 15);
        const int col = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(sQa + (row * PITCH + col) * 2, a0, a1, a2, a3);
      }
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        uint32_t b0, b1, b2, b3;
        const int mi = lane >> 3, r = lane & 7;
        const int key = nt * 8 + (mi >> 1) * 8 + r;
        const int col = kk * 16 + (mi & 1) * 8;
        ldsm_x4(sKa + (key * PITCH + col) * 2, b0, b1, b2, b3);
        mma_bf16_16816(s[nt], a0, a1, a2, a3, b0, b1);
        mma_bf16_16816(s[nt + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // mask + online softmax (base 2)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kj = nt * 8 + (lane & 3) * 2 + e;
        const int j = kb * ATT_BN + kj;
        const bool vis = sMask[buf * 64 + kj] != 0;
        const bool pre = j < p.n_prefix;
        const int kbv = sKb[buf * 64 + kj];
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
    const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
    const float base0 = (nm0 == -INFINITY) ? 0.f : nm0;
    const float base1 = (nm1 == -INFINITY) ? 0.f : nm1;
    const float c0 = exp2f(m0 - base0), c1 = exp2f(m1 - base1);
    m0 = nm0;
    m1 = nm1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - base0);
      s[nt][1] = exp2f(s[nt][1] - base0);
      s[nt][2] = exp2f(s[nt][2] - base1);
      s[nt][3] = exp2f(s[nt][3] - base1);
      rs0 += s[nt][0] + s[nt][1];
      rs1 += s[nt][2] + s[nt][3];
    }
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
#pragma unroll
    for (int i = 0; i < NT_D; ++i) {
      o[i][0] *= c0;
      o[i][1] *= c0;
      o[i][2] *= c1;
      o[i][3] *= c1;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a0 = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int nt = 0; nt < NT_D; nt += 2) {
        uint32_t b0, b1, b2, b3;
        const int mi = lane >> 3, r = lane & 7;
        const int key = kk * 16 + (mi & 1) * 8 + r;
        const int col = nt * 8 + (mi >> 1) * 8;
        ldsm_x4_t(sVa + (key * PITCH + col) * 2, b0, b1, b2, b3);
        mma_bf16_16816(o[nt], a0, a1, a2, a3, b0, b1);
        mma_bf16_16816(o[nt + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }

  // finalize: full row sums across the quad
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const int bh = b * p.heads + h;
  if (p.splits == 1) {
    const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
    const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
    bf16* go = p.o + (long long)b * p.q_br * p.o_rs + h * p.o_hs;
#pragma unroll
    for (int nt = 0; nt < NT_D; ++nt) {
      const int d = nt * 8 + (lane & 3) * 2;
      if (d < HD) {
        if (qr0 < p.n_q)
          *reinterpret_cast<uint32_t*>(go + (long long)qr0 * p.o_rs + d) =
              pack_bf16x2(o[nt][0] * inv0, o[nt][1] * inv0);
        if (qr1 < p.n_q)
          *reinterpret_cast<uint32_t*>(go + (long long)qr1 * p.o_rs + d) =
              pack_bf16x2(o[nt][2] * inv1, o[nt][3] * inv1);
      }
    }
  } else {
    const long long rows = (long long)p.batch * p.heads * p.n_q;
    float* po = p.part_o + ((long long)split * rows + (long long)bh * p.n_q) * HD;
    float* pml = p.part_ml + ((long long)split * rows + (long long)bh * p.n_q) * 2;
#pragma unroll
    for (int nt = 0; nt < NT_D; ++nt) {
      const int d = nt * 8 + (lane & 3) * 2;
      if (d < HD) {
        if (qr0 < p.n_q)
          *reinterpret_cast<float2*>(po + (long long)qr0 * HD + d) =
              make_float2(o[nt][0], o[nt][1]);
        if (qr1 < p.n_q)
          *reinterpret_cast<float2*>(po + (long long)qr1 * HD + d) =
              make_float2(o[nt][2], o[nt][3]);
      }
    }
    if ((lane & 3) == 0) {
      if (qr0 < p.n_q)
        *reinterpret_cast<float2*>(pml + (long long)qr0 * 2) =
            make_float2(m0, l0);
      if (qr1 < p.n_q)
        *reinterpret_cast<float2*>(pml + (long long)qr1 * 2) =
            make_float2(m1, l1);
    }
  }
}

// One CTA per (batch*head, query row), HD (or 96) threads: the split
// weights are computed once into shared memory, then every thread sums its
// dimension over the splits with independent loads.
constexpr int ATT_MAX_SPLITS = 64;
template <int HD>
__global__ void attn_combine_kernel(const AttnDev p) {
  __shared__ float w_s[ATT_MAX_SPLITS];
  __shared__ float inv_l;
  griddep_wait();
  griddep_launch_dependents();
  const int row = blockIdx.x;  // over batch*heads*n_q
  const int d = threadIdx.x;
  const long long rows = (long long)p.batch * p.heads * p.n_q;
  if (threadIdx.x < 32) {
    float m[2], l[2];
    float M = -INFINITY;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int s = threadIdx.x + 32 * i;
      m[i] = -INFINITY;
      l[i] = 0.f;
      if (s < p.splits) {
        const float2 ml = *reinterpret_cast<const float2*>(
            p.part_ml + ((long long)s * rows + row) * 2);
        m[i] = ml.x;
        l[i] = ml.y;
      }
      if (l[i] > 0.f) M = fmaxf(M, m[i]);
    }
    M = warp_max(M);
    float L = 0.f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int s = threadIdx.x + 32 * i;
      const float w = (l[i] > 0.f) ? exp2f(m[i] - M) : 0.f;
      if (s < ATT_MAX_SPLITS) w_s[s] = w;
      L += l[i] * w;
    }
    L = warp_sum(L);
    if (threadIdx.x == 0) inv_l = L > 0.f ? 1.f / L : 0.f;
  }
  __syncthreads();
  const int bh = row / p.n_q, r = row % p.n_q;
  const int b = bh / p.heads, h = bh % p.heads;
  if (d < HD) {
    float acc = 0.f;
    const float* po = p.part_o + (long long)row * HD + d;
#pragma unroll 8
    for (int s = 0; s < p.splits; ++s) acc += w_s[s] * po[(long long)s * rows * HD];
    bf16* go = p.o + ((long long)b * p.q_br + r) * p.o_rs + h * p.o_hs + d;
    *go = __float2bfloat16(acc * inv_l);
  }
}

template <int HD, int HDP>
constexpr int attn_smem_bytes() {
  return 5 * 64 * (HDP + 8) * 2 + 128 + 2 * 64 * 4;
}

}  // namespace fvb
