// Tensor-core (tcgen05 / TMEM) attention for the prefix prefill: SigLIP
// self-attention (head_dim 72, no mask) and the Gemma prefix (head_dim 256,
// MQA: 8 query heads on 1 K/V head, key padding mask).
//
// CTA = 128 query rows x all keys.  The rows of one K/V head's query group
// are flattened (row r -> query head r / n_q, query row r % n_q), so with MQA
// a tile spans heads and every CTA streams the shared K/V once.
//   warps 0-7 : softmax.  Warp w owns TMEM lanes 32*(w%4).. (query rows)
//               and key columns 32*(w/4).. of each 64-key block; the two
//               warps of a row exchange row maxima (and at the end row sums)
//               through shared memory.  They write Q (zero-padded to HDP)
//               into TMEM, read S = Q K^T from TMEM, write P (bf16) back
//               into the same TMEM columns, and finally read O, divide by
//               the row sum and store.
//   warp 8    : TMA producer of K tiles, warp 9 of V tiles (64 keys x 64
//               columns per box, 128-byte swizzle), KS stages each.
//   warp 10   : allocates TMEM and issues the MMAs from one lane, A operands
//               from TMEM, B operands from shared memory:
//               S(j) = Q K_j^T  (M=128, N=64, K=HDP; K tile K-major)
//               O   += P_j V_j  (M=128, N=NV, K=64; V is [key][dim] in
//               memory, i.e. MN-major for the B operand)
//               S(j+1) is issued before O += P_j V_j so the softmax of block
//               j overlaps the next QK^T.  MMAs of one thread execute in
//               order, so S(j+2) overwriting the P(j) columns follows PV(j).
// TMEM (32-bit columns): O [0, NV), S/P buffers 2 x 64, Q HDP/2 (bf16 pairs).
// Keeping Q and P in TMEM leaves shared memory to the K/V pipeline.
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
#include "gemm_tc.cuh"  // g_gemm_trace (diagnostic stamps)

namespace fvb {
namespace atc {

constexpr int BM = 128, BKV = 64, THREADS = 352;

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
  int trace;                 // diagnostics: per-block stamps of CTA (0,0,0)
  // split over keys (splits > 1): blockIdx.z = batch * splits + split covers
  // key blocks [split * blocks_per_split, ...) and writes its un-normalised
  // partial (O f32, max, sum) for attn_combine_kernel
  int heads, splits, blocks_per_split;
  float* part_o;   // [splits][batch*heads*n_q][HD]
  float* part_ml;  // [splits][batch*heads*n_q][2]
};

// keys per launch covered by the shared-memory validity bitmask
constexpr int MAX_KEYS = 1024;
constexpr int SOFTMAX_WARPS = 8;

template <int HD, int HDP, int NV>
struct AtcCfg {
  static_assert(HDP % 64 == 0 && HD <= HDP && NV % 16 == 0 && NV >= HD &&
                    NV <= 256,
                "shape");
  static constexpr int K_BYTES = BKV * HDP * 2;
  static constexpr int V_CHUNKS = (NV + 63) / 64;
  static constexpr int V_BYTES = BKV * V_CHUNKS * 128;
  static constexpr int KS = (200 * 1024) / (K_BYTES + V_BYTES) < 4
                                ? (200 * 1024) / (K_BYTES + V_BYTES) : 4;
  static_assert(KS >= 2, "K/V stages");
  static constexpr int OFF_V = KS * K_BYTES;
  static constexpr int OFF_X = OFF_V + KS * V_BYTES;  // [2 parity][2 halves][BM] f32
  static constexpr int OFF_MASK = OFF_X + 2 * 2 * BM * 4;
  static constexpr int OFF_BAR = OFF_MASK + MAX_KEYS / 8;
  static constexpr int SMEM = OFF_BAR + 512 + 1024;
  static constexpr uint32_t TMEM_S = NV <= 128 ? 128u : 256u;  // 2 x BKV
  static constexpr uint32_t TMEM_Q = TMEM_S + 2 * BKV;         // HDP / 2
  static_assert(TMEM_Q + HDP / 2 <= 512, "TMEM");
  static constexpr uint32_t TMEM_COLS = TMEM_Q + HDP / 2 <= 256 ? 256u : 512u;
};

__device__ __forceinline__ void atc_stamp(const AtcDev& p, int row, int slot) {
  if (p.trace && row < 64 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
    g_gemm_trace[row][slot] = globaltimer_ns();
}

template <int HD, int HDP, int NV>
__global__ void __launch_bounds__(THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AtcDev p) {
  using C = AtcCfg<HD, HDP, NV>;
  constexpr int KS = C::KS;
  constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BKV);
  constexpr uint32_t IDESC_PV = idesc_bf16_f32(BM, NV) | (1u << 16);  // B MN-major
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + C::OFF_V;
  float* sX = reinterpret_cast<float*>(smem + C::OFF_X);
  uint32_t* sMask = reinterpret_cast<uint32_t*>(smem + C::OFF_MASK);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* k_full = bars;             // [KS]
  uint64_t* k_empty = bars + KS;       // [KS]
  uint64_t* v_full = bars + 2 * KS;    // [KS]
  uint64_t* v_empty = bars + 3 * KS;   // [KS]
  uint64_t* q_full = bars + 4 * KS;
  uint64_t* s_full = q_full + 1;       // [2]
  uint64_t* p_full = q_full + 3;       // [2]
  uint64_t* o_done = q_full + 5;       // [2]
  uint64_t* o_final = q_full + 7;
  uint64_t* x_bar = q_full + 8;        // [2] row-max exchange, block j -> j&1
  uint64_t* m_bar = q_full + 10;       // key bitmask built
  uint64_t* l_bar = q_full + 11;       // row-sum exchange
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_full + 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, kvh = blockIdx.y;
  const int b = blockIdx.z / p.splits, split = blockIdx.z % p.splits;
  const int nkb_all = (p.n_kv + BKV - 1) / BKV;
  const int kb_begin = split * p.blocks_per_split;
  const int nkb = min(p.blocks_per_split, nkb_all - kb_begin);  // this CTA's blocks
  // Key blocks are visited in the order kb0, kb0+1, ... (mod nkb), kb0
  // different per query tile, so the tiles of one K/V head do not all read
  // the same K/V lines at the same moment (the online softmax does not
  // depend on the order).
  const int kb0 = tile % nkb;
  auto key_block = [&](int j) {
    const int k = j + kb0;
    return kb_begin + (k >= nkb ? k - nkb : k);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(q_full, SOFTMAX_WARPS);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], SOFTMAX_WARPS);
      mbar_init(&o_done[s], 1);
      mbar_init(&x_bar[s], SOFTMAX_WARPS);
    }
    mbar_init(o_final, 1);
    mbar_init(m_bar, SOFTMAX_WARPS);
    mbar_init(l_bar, SOFTMAX_WARPS);
    fence_barrier_init();
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
  }
  if (warp == 10) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 8 || warp == 9) {
    // K (warp 8) or V (warp 9) producer
    if (lane == 0) {
      const bool is_k = warp == 8;
      const CUtensorMap* map = is_k ? &tmK : &tmV;
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      uint8_t* dst = is_k ? sK : sV;
      const int bytes = is_k ? C::K_BYTES : C::V_BYTES;
      const int chunks = is_k ? HDP / 64 : C::V_CHUNKS;
      const int x0 = kvh * (is_k ? p.k_hs : p.v_hs);
      const int y0 = (int)((long long)b * p.kv_br);
      for (int j = 0; j < nkb; ++j) {
        const int s = j % KS;
        if (!mbar_wait(&empty[s], ((j / KS) & 1) ^ 1)) break;
        atc_stamp(p, j, is_k ? 6 : 7);
        mbar_arrive_expect_tx(&full[s], bytes);
        for (int c = 0; c < chunks; ++c)
          tma_load_2d(dst + s * bytes + c * BKV * 128, map, x0 + c * 64,
                      y0 + key_block(j) * BKV, &full[s]);
      }
    }
  } else if (warp == 10) {
    if (lane == 0) {
      bool alive = mbar_wait_spin(q_full, 0);
      atc_stamp(p, 63, 2);
      tc_fence_after();
      auto issue_s = [&](int j) -> bool {
        const int ks = j % KS, sb = j & 1;
        if (!mbar_wait_spin(&k_full[ks], (j / KS) & 1)) return false;
        if (j == 0) atc_stamp(p, 63, 3);
        tc_fence_after();
        const uint32_t k_base = smem_u32(sK + ks * C::K_BYTES);
        const uint32_t d = tmem + C::TMEM_S + (uint32_t)(sb * BKV);
#pragma unroll
        for (int kk = 0; kk < HDP / 16; ++kk)
          tc_mma_bf16_ts(d, tmem + C::TMEM_Q + (uint32_t)(kk * 8),
                         smem_desc_sw128(k_base + (kk >> 2) * (BKV * 128) + (kk & 3) * 32),
                         IDESC_S, kk > 0 ? 1u : 0u);
        tc_commit(&s_full[sb]);
        tc_commit(&k_empty[ks]);
        atc_stamp(p, j, 4);
        return true;
      };
      if (alive) alive = issue_s(0);
      for (int j = 0; j < nkb && alive; ++j) {
        if (j + 1 < nkb && !(alive = issue_s(j + 1))) break;
        const int ks = j % KS, sb = j & 1;
        if (!mbar_wait_spin(&p_full[sb], (j >> 1) & 1) ||
            !mbar_wait_spin(&v_full[ks], (j / KS) & 1)) {
          alive = false;
          break;
        }
        tc_fence_after();
        atc_stamp(p, j, 5);
        const uint32_t v_base = smem_u32(sV + ks * C::V_BYTES);
        const uint32_t p_cols = tmem + C::TMEM_S + (uint32_t)(sb * BKV);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          tc_mma_bf16_ts(tmem, p_cols + (uint32_t)(kk * 8),
                         smem_desc_sw128_mn(v_base + kk * 2048, BKV * 128),
                         IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&o_done[sb]);
        tc_commit(&v_empty[ks]);
      }
      if (alive) tc_commit(o_final);
    }
  } else {
    // ---- softmax warps: query row i, key columns [32*hf, 32*hf + 32) ----
    const int qd = warp & 3, hf = warp >> 2;
    const int i = qd * 32 + lane;
    const int tid = hf * BM + i;  // 0..255 over the softmax warps
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const int rows_total = p.group * p.n_q;
    const int r = tile * BM + i;
    const bool row_ok = r < rows_total;
    const int h = kvh * p.group + (row_ok ? r / p.n_q : 0);
    const int qrow = row_ok ? r % p.n_q : 0;
    {
      // Q row i, bf16 pairs [hf*HDP/4, (hf+1)*HDP/4) -> TMEM columns
      const bf16* gq = p.q + ((long long)b * p.q_br + qrow) * p.q_rs + (long long)h * p.q_hs;
      constexpr int QW = HDP / 4;  // 32-bit words of this half row
#pragma unroll 1
      for (int w0 = 0; w0 < QW; w0 += 16) {
        uint32_t q[16];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = (hf * QW + w0 + 4 * u) * 2;  // first element of the chunk
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (row_ok && e < HD) v = *reinterpret_cast<const uint4*>(gq + e);
          q[4 * u] = v.x; q[4 * u + 1] = v.y; q[4 * u + 2] = v.z; q[4 * u + 3] = v.w;
        }
        tmem_st16(tmem + lane_base + C::TMEM_Q + (uint32_t)(hf * QW + w0), q);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_full);
      if (tid == 0) atc_stamp(p, 63, 0);
    }
    // key validity bitmask of all blocks (bit t of word w = key 32w + t)
    for (int w = tid; w < nkb_all * 2; w += 2 * BM) {
      uint32_t bits = 0;
#pragma unroll 8
      for (int t = 0; t < 32; ++t) {
        const int key = w * 32 + t;
        bool ok = key < p.n_kv;
        if (ok && p.key_valid) ok = p.key_valid[key] != 0;
        bits |= (ok ? 1u : 0u) << t;
      }
      sMask[w] = bits;
    }
    // the softmax warps exchange data through mbarriers with bounded waits
    // (a warp that gives up cannot leave the others blocked)
    __syncwarp();
    if (lane == 0) mbar_arrive(m_bar);
    bool alive = __all_sync(0xffffffffu, mbar_wait_spin(m_bar, 0));
    if (tid == 0) atc_stamp(p, 63, 1);

    float m_ref = -INFINITY, l = 0.f;
    for (int j = 0; j < nkb && alive; ++j) {
      const int sb = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      const uint32_t kv = sMask[2 * key_block(j) + hf];
      const uint32_t s_cols = tmem + lane_base + C::TMEM_S + (uint32_t)(sb * BKV);
      if (!__all_sync(0xffffffffu, mbar_wait_spin(&s_full[sb], ph))) { alive = false; break; }
      tc_fence_after();
      if (tid == 0) atc_stamp(p, j, 0);
      uint32_t ra[32];
      tmem_ld32(s_cols + (uint32_t)(hf * 32), ra);
      tmem_wait_ld32(ra);
      if (tid == 0) atc_stamp(p, j, 1);
      float x[32];
      float pm = -INFINITY;
#pragma unroll
      for (int t = 0; t < 32; ++t) {
        x[t] = ((kv >> t) & 1u) ? __uint_as_float(ra[t]) * p.scale_log2 : -INFINITY;
        pm = fmaxf(pm, x[t]);
      }
      // row max over both column halves.  The P of this half is computed
      // against the current reference while the exchange completes and is
      // recomputed only if some row of the warp raises the reference.
      // The arrive also orders this warp's S reads before the partner
      // warp's P writes into the same columns.
      float* xs = sX + sb * (2 * BM);
      xs[hf * BM + i] = pm;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&x_bar[sb]);
      uint32_t pw[16];
      float rs = 0.f;
      auto make_p = [&](float ref) {
        const float base = (ref == -INFINITY) ? 0.f : ref;
        rs = 0.f;
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const float p0 = exp2f(x[t] - base), p1 = exp2f(x[t + 1] - base);
          rs += p0 + p1;
          pw[t >> 1] = pack_bf16x2(p0, p1);
        }
      };
      make_p(m_ref);  // block 0: recomputed below unless every key is masked
      if (!__all_sync(0xffffffffu, mbar_wait_spin(&x_bar[sb], ph))) { alive = false; break; }
      tc_fence_after();
      const float mx = fmaxf(pm, xs[(hf ^ 1) * BM + i]);
      // raise the reference max (warp-uniform decision; both warps of a row
      // pair see the same maxima and decide alike)
      const bool raise = mx > m_ref + 8.f;
      if (__any_sync(0xffffffffu, raise)) {
        const float nref = raise ? mx : m_ref;
        const float alpha = (m_ref == -INFINITY) ? 0.f : exp2f(m_ref - nref);
        if (j > 0) {
          // O holds blocks < j: wait for the last PV, rescale this warp's
          // 16-column chunks of O in place
          if (!__all_sync(0xffffffffu, mbar_wait_spin(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1))) {
            alive = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = hf * 16; c < NV; c += 32) {
            uint32_t o[16];
            tmem_ld16_sync(tmem + lane_base + (uint32_t)c, o);
#pragma unroll
            for (int t = 0; t < 16; ++t)
              o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
            tmem_st16(tmem + lane_base + (uint32_t)c, o);
          }
        }
        l *= alpha;
        m_ref = nref;
        make_p(m_ref);
      }
      l += rs;
      if (tid == 0) atc_stamp(p, j, 2);
      // P (bf16 pairs, keys in order) over this half's S columns
      tmem_st16(s_cols + (uint32_t)(hf * 16), pw);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
      if (tid == 0) atc_stamp(p, j, 3);
    }
    // ---- output: O / l, l summed over both column halves ----
    // row sums go through the max-exchange slots of parity (nkb-1)^1: those
    // were last read in block nkb-2, before every warp arrived on the
    // exchange barrier of block nkb-1
    float* ls = sX + (((nkb - 1) & 1) ^ 1) * (2 * BM);
    if (alive) {
      ls[hf * BM + i] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(l_bar);
      alive = __all_sync(0xffffffffu, mbar_wait_spin(l_bar, 0));
    }
    const float lt = alive ? l + ls[(hf ^ 1) * BM + i] : 0.f;
    if (alive && p.splits > 1 && __all_sync(0xffffffffu, mbar_wait_spin(o_final, 0))) {
      // partial: O relative to m_ref (f32), (m_ref, row sum)
      tc_fence_after();
      const long long rows = (long long)gridDim.z / p.splits * p.heads * p.n_q;
      const long long row = ((long long)b * p.heads + h) * p.n_q + qrow;
      float* po = p.part_o + ((long long)split * rows + row) * HD;
#pragma unroll 1
      for (int c = hf * 16; c < NV; c += 32) {
        uint32_t o[16];
        tmem_ld16_sync(tmem + lane_base + (uint32_t)c, o);
        if (row_ok) {
#pragma unroll
          for (int t = 0; t < 16; t += 4)
            if (c + t < HD)
              *reinterpret_cast<float4*>(po + c + t) =
                  make_float4(__uint_as_float(o[t]), __uint_as_float(o[t + 1]),
                              __uint_as_float(o[t + 2]), __uint_as_float(o[t + 3]));
        }
      }
      if (row_ok && hf == 0)
        *reinterpret_cast<float2*>(p.part_ml + ((long long)split * rows + row) * 2) =
            make_float2(m_ref, lt);
    } else if (alive && __all_sync(0xffffffffu, mbar_wait_spin(o_final, 0))) {
      tc_fence_after();
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      bf16* go = p.o + ((long long)b * p.q_br + qrow) * p.o_rs + (long long)h * p.o_hs;
#pragma unroll 1
      for (int c = hf * 16; c < NV; c += 32) {
        uint32_t o[16];
        tmem_ld16_sync(tmem + lane_base + (uint32_t)c, o);
        if (row_ok) {
#pragma unroll
          for (int t = 0; t < 16; t += 8) {
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
  if (warp == 10) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace atc
}  // namespace fvb
