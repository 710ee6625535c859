// Tensor-core (tcgen05 / TMEM) attention for the prefix prefill: SigLIP
// self-attention (head_dim 72, no mask) and the Gemma prefix (head_dim 256,
// MQA: 8 query heads on 1 K/V head, key padding mask).
//
// CTA = 128 query rows x all keys.  The rows of one K/V head's query group
// are flattened (row r -> query head r / n_q, query row r % n_q), so with MQA
// a tile spans heads and every CTA streams the shared K/V once.
//   warps 0-3 : softmax; thread i owns query row i = TMEM lane i.  They
//               stage Q (zero-padded to HDP columns) in shared memory, read
//               S = Q K^T rows from TMEM, write P (bf16) to shared memory,
//               and finally read O from TMEM, divide by the row sum, store.
//   warp 4    : TMA producer, K and V tiles of 64 keys, double-buffered
//               (boxes of 64 columns x 64 keys, 128-byte swizzle).
//   warp 5    : allocates TMEM and issues the MMAs from one lane:
//               S(j) = Q K_j^T  (M=128, N=64, K=HDP; both operands K-major)
//               O   += P_j V_j  (M=128, N=NV, K=64; V is [key][dim] in
//               memory, i.e. MN-major for the B operand)
//               S(j+1) is issued before O += P_j V_j so the softmax of block
//               j overlaps the next QK^T.
// TMEM: O in columns [0, NV), two S buffers of 64 columns after it.
//
// Online softmax with a lazily raised reference max: P = exp2(s - m_ref)
// with m_ref the running row max, raised (and O, l rescaled in place) only
// when a block's max exceeds m_ref by more than 8 (log2 units), so P stays
// below 2^8 and most blocks need no O rescale.  O and l always refer to the
// same m_ref, so the result is the exact softmax; the rescale decision is
// warp-uniform because tcgen05.ld / st are warp-collective.
//
// Semantics (same as attn_kernel): per query head, softmax over the valid
// keys of (Q K^T) * scale, times V; a row with no valid key outputs zeros.
#pragma once

#include "common.cuh"

namespace fvb {
namespace atc {

constexpr int BM = 128, BKV = 64, THREADS = 192;

struct AtcDev {
  const bf16* q;
  long long q_rs, q_hs;
  bf16* o;
  long long o_rs, o_hs;
  int k_hs, v_hs;  // column offset of a K/V head in the K/V tensor maps
  int n_q, n_kv, group;
  long long q_br, kv_br;
  float scale_log2;
  const uint8_t* key_valid;  // [n_kv] or null
};

template <int HD, int HDP, int NV>
struct AtcCfg {
  static_assert(HDP % 64 == 0 && HD <= HDP && NV % 16 == 0 && NV >= HD &&
                    NV <= 256,
                "shape");
  static constexpr int Q_BYTES = BM * HDP * 2;
  static constexpr int K_BYTES = BKV * HDP * 2;
  static constexpr int V_CHUNKS = (NV + 63) / 64;
  static constexpr int V_BYTES = BKV * V_CHUNKS * 128;
  static constexpr int P_BYTES = BM * BKV * 2;
  static constexpr int OFF_K = Q_BYTES;
  static constexpr int OFF_V = OFF_K + 2 * K_BYTES;
  static constexpr int OFF_P = OFF_V + 2 * V_BYTES;
  static constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static constexpr uint32_t TMEM_S = NV <= 128 ? 128u : 256u;
  static constexpr uint32_t TMEM_COLS = TMEM_S + 2 * BKV <= 256 ? 256u : 512u;
};

// K-major SW128 descriptor = smem_desc_sw128.  MN-major SW128 (the V
// operand): 64 MN-elements (128 B) per row, one row per K index, 8-row
// groups 1024 B apart (stride byte offset), MN atoms `lbo` bytes apart
// (leading byte offset).
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(uint32_t saddr,
                                                       uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
      "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]),
      "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
      "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

template <int HD, int HDP, int NV>
__global__ void __launch_bounds__(THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AtcDev p) {
  using C = AtcCfg<HD, HDP, NV>;
  constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BKV);
  constexpr uint32_t IDESC_PV = idesc_bf16_f32(BM, NV) | (1u << 16);  // B MN-major
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + C::OFF_K;
  uint8_t* sV = smem + C::OFF_V;
  uint8_t* sP = smem + C::OFF_P;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [2]
  uint64_t* s_free = bars + 11;   // [2]
  uint64_t* p_full = bars + 13;   // [2]
  uint64_t* o_done = bars + 15;   // [2]
  uint64_t* o_final = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int nkb = (p.n_kv + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 4);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 4);
      mbar_init(&p_full[s], 4);
      mbar_init(&o_done[s], 1);
    }
    mbar_init(o_final, 1);
    fence_barrier_init();
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
  }
  if (warp == 5) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 4) {
    if (lane == 0) {
      const int y0 = (int)((long long)b * p.kv_br);
      for (int j = 0; j < nkb; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_empty[s], ph ^ 1)) break;
        mbar_arrive_expect_tx(&k_full[s], C::K_BYTES);
#pragma unroll
        for (int c = 0; c < HDP / 64; ++c)
          tma_load_2d(sK + s * C::K_BYTES + c * BKV * 128, &tmK,
                      kvh * p.k_hs + c * 64, y0 + j * BKV, &k_full[s]);
        if (!mbar_wait(&v_empty[s], ph ^ 1)) break;
        mbar_arrive_expect_tx(&v_full[s], C::V_BYTES);
#pragma unroll
        for (int c = 0; c < C::V_CHUNKS; ++c)
          tma_load_2d(sV + s * C::V_BYTES + c * BKV * 128, &tmV,
                      kvh * p.v_hs + c * 64, y0 + j * BKV, &v_full[s]);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      bool alive = mbar_wait(q_full, 0);
      tc_fence_after();
      const uint32_t q_base = smem_u32(sQ);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&k_full[s], (j >> 1) & 1)) return false;
        if (j >= 2 && !mbar_wait(&s_free[s], ((j - 2) >> 1) & 1)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_u32(sK + s * C::K_BYTES);
        const uint32_t d = tmem + C::TMEM_S + (uint32_t)(s * BKV);
#pragma unroll
        for (int kk = 0; kk < HDP / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk & 3) * 32);
          tc_mma_bf16(d, smem_desc_sw128(q_base + (kk >> 2) * (BM * 128) + off),
                      smem_desc_sw128(k_base + (kk >> 2) * (BKV * 128) + off),
                      IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[s]);
        tc_commit(&k_empty[s]);
        return true;
      };
      if (alive) alive = issue_s(0);
      for (int j = 0; j < nkb && alive; ++j) {
        if (j + 1 < nkb && !(alive = issue_s(j + 1))) break;
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&p_full[s], ph) || !mbar_wait(&v_full[s], ph)) {
          alive = false;
          break;
        }
        tc_fence_after();
        const uint32_t p_base = smem_u32(sP + s * C::P_BYTES);
        const uint32_t v_base = smem_u32(sV + s * C::V_BYTES);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          tc_mma_bf16(tmem, smem_desc_sw128(p_base + kk * 32),
                      smem_desc_sw128_mn(v_base + kk * 2048, BKV * 128),
                      IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&o_done[s]);
        tc_commit(&v_empty[s]);
      }
      if (alive) tc_commit(o_final);
    }
  } else {
    // ---- softmax warps: thread = query row i ----
    const int i = warp * 32 + lane;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const int rows_total = p.group * p.n_q;
    const int r = tile * BM + i;
    const bool row_ok = r < rows_total;
    const int h = kvh * p.group + (row_ok ? r / p.n_q : 0);
    const int qrow = row_ok ? r % p.n_q : 0;
    {
      const bf16* gq = p.q + ((long long)b * p.q_br + qrow) * p.q_rs + (long long)h * p.q_hs;
      const uint32_t q_base = smem_u32(sQ);
#pragma unroll 4
      for (int c = 0; c < HDP / 8; ++c) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (row_ok && c * 8 < HD) v = *reinterpret_cast<const uint4*>(gq + c * 8);
        const int a = c >> 3, cc = c & 7;
        const uint32_t addr = q_base + a * (BM * 128) + i * 128 + ((cc ^ (i & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr),
                     "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_full);
    }
    float m_ref = -INFINITY, l = 0.f;
    bool alive = true;
    const uint32_t p_row = (uint32_t)(i * 128);
    for (int j = 0; j < nkb; ++j) {
      const int s = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      // key validity of this block: bit t of kv[t / 32]
      const int key0 = j * BKV;
      uint32_t kv[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int key = key0 + hh * 32 + lane;
        bool ok = key < p.n_kv;
        if (ok && p.key_valid) ok = p.key_valid[key] != 0;
        kv[hh] = __ballot_sync(0xffffffffu, ok);
      }
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[s], ph))) { alive = false; break; }
      tc_fence_after();
      uint32_t ra[32], rb[32];
      tmem_ld32(tmem + lane_base + C::TMEM_S + (uint32_t)(s * BKV), ra);
      tmem_ld32(tmem + lane_base + C::TMEM_S + (uint32_t)(s * BKV + 32), rb);
      tmem_wait_ld32(ra);
      tmem_wait_ld32(rb);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[s]);
      float x[64];
      float mx = -INFINITY;
#pragma unroll
      for (int t = 0; t < 32; ++t) {
        x[t] = ((kv[0] >> t) & 1u) ? __uint_as_float(ra[t]) * p.scale_log2 : -INFINITY;
        x[32 + t] = ((kv[1] >> t) & 1u) ? __uint_as_float(rb[t]) * p.scale_log2 : -INFINITY;
        mx = fmaxf(mx, fmaxf(x[t], x[32 + t]));
      }
      // raise the reference max (warp-uniform decision)
      const bool raise = mx > m_ref + 8.f;
      if (__any_sync(0xffffffffu, raise)) {
        const float nref = raise ? mx : m_ref;
        const float alpha = (m_ref == -INFINITY) ? 0.f : exp2f(m_ref - nref);
        if (j > 0) {
          // O holds blocks < j: wait for the last PV, rescale in place
          if (!__all_sync(0xffffffffu, mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1))) {
            alive = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < NV; c += 32) {
            uint32_t o[32];
            tmem_ld32(tmem + lane_base + (uint32_t)c, o);
            tmem_wait_ld32(o);
#pragma unroll
            for (int t = 0; t < 32; ++t)
              o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
            tmem_st32(tmem + lane_base + (uint32_t)c, o);
          }
          tmem_wait_st();
        }
        l *= alpha;
        m_ref = nref;
      }
      const float base = (m_ref == -INFINITY) ? 0.f : m_ref;
      uint32_t pw[32];
      float rs = 0.f;
#pragma unroll
      for (int t = 0; t < 64; t += 2) {
        const float p0 = exp2f(x[t] - base), p1 = exp2f(x[t + 1] - base);
        rs += p0 + p1;
        pw[t >> 1] = pack_bf16x2(p0, p1);
      }
      l += rs;
      // P buffer s is free once PV(j-2) has completed
      if (j >= 2 && !__all_sync(0xffffffffu, mbar_wait(&o_done[s], ((j - 2) >> 1) & 1))) {
        alive = false;
        break;
      }
      const uint32_t pb = smem_u32(sP + s * C::P_BYTES);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t addr = pb + p_row + ((c ^ (i & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr),
                     "r"(pw[4 * c]), "r"(pw[4 * c + 1]), "r"(pw[4 * c + 2]),
                     "r"(pw[4 * c + 3])
                     : "memory");
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[s]);
    }
    // ---- output: O / l ----
    if (alive && __all_sync(0xffffffffu, mbar_wait(o_final, 0))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* go = p.o + ((long long)b * p.q_br + qrow) * p.o_rs + (long long)h * p.o_hs;
#pragma unroll 1
      for (int c = 0; c < NV; c += 32) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + (uint32_t)c, o);
        tmem_wait_ld32(o);
        if (row_ok) {
#pragma unroll
          for (int t = 0; t < 32; t += 8) {
            if (c + t < HD) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(o[t]) * inv, __uint_as_float(o[t + 1]) * inv);
              w.y = pack_bf16x2(__uint_as_float(o[t + 2]) * inv, __uint_as_float(o[t + 3]) * inv);
              w.z = pack_bf16x2(__uint_as_float(o[t + 4]) * inv, __uint_as_float(o[t + 5]) * inv);
              w.w = pack_bf16x2(__uint_as_float(o[t + 6]) * inv, __uint_as_float(o[t + 7]) * inv);
              *reinterpret_cast<uint4*>(go + c + t) = w;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace atc
}  // namespace fvb
