// Two-SM (cta_group::2) tensor-core GEMM, swapped orientation:
//   out[token, feature] (op)= sum_k W[feature, k] * X[token, k]
// for the big prefill projections whose weight side is wide (Gemma gate/up
// 32768 rows, down 2048 rows) and whose token side is the 816-row prefix.
//
// A CTA pair (a 2-CTA cluster) owns a 256-weight-row x BN-token tile: each
// CTA loads its own 128 weight rows (A) and half of the BN token rows (B)
// per 64-wide k step, and the leader CTA issues tcgen05.mma.cta_group::2
// (M = 256, N = BN) which reads A and B from both CTAs' shared memory and
// accumulates rows 0..127 in the leader's TMEM and 128..255 in the peer's.
// Per SM this moves (128 + BN/2) rows of operands for 128 x BN of output,
// half the token traffic of a one-SM 128 x BN tile — the per-SM L2->shared
// operand stream is what bounds the one-SM kernel on these shapes.
//
//   warp 0 (one lane, both CTAs): TMA producer; its loads complete on the
//          leader's full[] barrier (the leader posts the expected bytes of
//          both CTAs), its stages are freed by the leader's multicast commit
//   warp 1 (one lane, leader only): tcgen05.mma.cta_group::2 issuer
//   warps 2..5 (both CTAs): epilogue from the CTA's own TMEM lanes (its 128
//          weight rows) through shared-memory staging and TMA stores /
//          reduce-adds, then a release-arrive on the leader's tempty[]
// Two TMEM accumulators of BN columns per CTA; TMA loads without multicast.
#pragma once

#include "gemm_tc.cuh"

namespace fvb {
namespace pair {

constexpr int THREADS = 192;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void tmem_alloc2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst_smem)),
      "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr),
               "r"(ncols));
}
__device__ __forceinline__ void mma2_bf16(uint32_t tmem_d, uint64_t adesc,
                                          uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// arrive on the barrier at this shared offset in both CTAs of the pair once
// the issuing thread's prior MMAs are complete
__device__ __forceinline__ void commit2_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster."
      "multicast::cluster.b64 [%0], %1;" ::"r"(smem_u32(bar)),
      "h"((unsigned short)0x3)
      : "memory");
}
// TMA tile load into this CTA's shared memory, completing on the mbarrier at
// shared::cluster address `bar_cluster` (the leader's barrier)
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map,
                                                 int32_t x, int32_t y,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::"
      "complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                   bar_cluster)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait with cluster-scope acquire (arrivals come from the peer CTA)
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t n = 0;; ++n) {
    if (mbar_try_wait_cluster(addr, parity)) return true;
    if ((n & 63) == 63 && globaltimer_ns() - t0 > FVB_WAIT_LIMIT_NS) {
      record_device_error(FVB_ERR_DEVICE_TIMEOUT);
      return false;
    }
  }
}

// Per epilogue warp: two staging slots of two boxes each; a box holds 16
// token rows of 32 f32 features (128-byte rows) or of 16 bf16 GeGLU outputs
// (32-byte rows, packed)
constexpr int STG_BOX = 16 * 128;
constexpr int STG_SLOT = 2 * STG_BOX;
constexpr int STG_WARP = 2 * STG_SLOT;

template <int BN>
struct PairCfg {
  static_assert(BN % 16 == 0 && (BN / 2) % 8 == 0 && BN >= 64 && BN <= 256, "block_n");
  static constexpr int A_BYTES = 128 * GEMM_BK * 2;
  static constexpr int B_BYTES = (BN / 2) * GEMM_BK * 2;  // this CTA's half
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (184 * 1024) / STAGE_BYTES < 8 ? (184 * 1024) / STAGE_BYTES : 8;
  static constexpr int OFF_STG = STAGES * STAGE_BYTES;  // 1024-aligned
  static constexpr int OFF_BAR = OFF_STG + 4 * STG_WARP;
  static constexpr int SMEM = OFF_BAR + 1024 + 256;
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 256 ? 256u : 512u;
  static constexpr uint32_t ACC_STRIDE = TMEM_COLS / 2;  // accumulator columns
};

// Epilogue of one accumulator through TMA: thread = weight row (its TMEM
// lane), 32 token columns per step (the next step's TMEM load in flight
// while this one is staged), written as 16-token boxes.
//   GEGLU:   rows 2i / 2i+1 are gate / up of output feature i; the lane pair
//            exchanges half its columns so that each lane finishes 16 tokens,
//            h[token, i] = gelu(gate) * up, TMA tile store (bf16).
//   F32_ACC: out[token, f] += (acc + bias[f]) * gate[f] * alpha, TMA f32
//            reduce-add (also merges K splits in L2).
// Boxes of tokens past this tile or past n are not issued; the tensor map
// clips features past m.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_pair(const GemmDev& p, const CUtensorMap* tmO,
                                              uint32_t taddr, uint8_t* stg, int f0,
                                              int bcol0, int split, int lane, int& uses) {
  const int n_tok = p.n;
  float fb = 0.f, fg = 1.f;
  if (EPI == FVB_EPI_F32_ACC) {
    const int fs = min(f0 + lane, p.m - 1);
    fb = (p.bias != nullptr && split == 0) ? __ldg(p.bias + fs) : 0.f;
    fg = p.alpha * (p.gate ? __ldg(p.gate + fs) : 1.f);
  }
  uint32_t ra[32];
  tmem_ld32(taddr, ra);
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    const int t0 = bcol0 + c;
    float v[32];
    tmem_wait_ld32(ra);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(ra[j]);
    const bool more = c + 32 < BN && t0 + 32 < n_tok;  // uniform
    if (more) tmem_ld32(taddr + (uint32_t)(c + 32), ra);
    const int nb = (c + 16 < BN && t0 + 16 < n_tok) ? 2 : 1;
    uint8_t* slot = stg + (uses & 1) * STG_SLOT;
    if (lane == 0) bulk_wait_read1();  // the store that last read this slot
    __syncwarp();
    if (EPI == FVB_EPI_GEGLU) {
      const bool odd = lane & 1;
      float rc[16];
#pragma unroll
      for (int j = 0; j < 16; ++j)
        rc[j] = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[16 + j], 1);
      // even lane: tokens 0..15 (gate v, up from the odd lane); odd lane:
      // tokens 16..31 (gate from the even lane, up v)
      bf16* box = reinterpret_cast<bf16*>(slot + (odd ? STG_BOX : 0));
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float g = odd ? rc[j] : v[j];
        const float u = odd ? v[16 + j] : rc[j];
        box[j * 16 + (lane >> 1)] = __float2bfloat16(gelu_tanh_f(g) * u);
      }
    } else {
      float* box = reinterpret_cast<float*>(slot);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        box[(j >> 4) * (STG_BOX / 4) + (j & 15) * 32 + lane] = (v[j] + fb) * fg;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      for (int b = 0; b < nb; ++b) {
        if (EPI == FVB_EPI_GEGLU)
          tma_store_2d(tmO, f0 >> 1, t0 + 16 * b, slot + b * STG_BOX);
        else
          tma_reduce_add_2d(tmO, f0, t0 + 16 * b, slot + b * STG_BOX);
      }
      bulk_commit();
    }
    ++uses;
  }
}

// Work item w of the pairs: token tile fastest, then weight row pair tile
// (256 rows, m_tiles counts them), then K split.  The pairs running at one
// time then share a few weight tiles across all token tiles, so each weight
// byte comes from HBM once (a weight-fastest order re-streams the whole
// weight matrix, larger than L2, once per token tile).
__device__ __forceinline__ Tile decode_pair_tile(const GemmDev& p, int w) {
  Tile t;
  t.nt = w % p.n_tiles;
  const int rest = w / p.n_tiles;
  t.m0 = (rest % p.m_tiles) * GEMM_BM;
  t.split = rest / p.m_tiles;
  t.kt0 = t.split * p.kt_per_split;
  t.kt1 = min(t.kt0 + p.kt_per_split, p.k_tiles);
  return t;
}

template <int BN, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmO, const GemmDev p) {
  using Cfg = PairCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = idesc_bf16_f32(256, BN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2]
  uint64_t* tempty = tfull + 2;      // [2] (leader: 4 warps x 2 CTAs)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  // diagnostics (launch made with tracing on): [0] start, [1] set up, per
  // tile j < 3: [2+4j] first k-tile landed (MMA issuer), [3+4j] accumulator
  // committed, [4+4j] epilogue start, [5+4j] epilogue done; [14] end
  trace_stamp(p, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    fence_barrier_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    prefetch_tensormap(&tmO);
  }
  if (warp == 1) tmem_alloc2(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) trace_stamp(p, 1);
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int w = pair; w < p.n_work; w += n_pairs) {
        const Tile t = decode_pair_tile(p, w);
        const int wrow = (t.m0 << 1) + (int)rank * 128;  // m0 = 128 * pair tile
        const int trow = t.nt * BN + (int)rank * (BN / 2);
        bool alive = true;
        for (int kt = t.kt0; kt < t.kt1; ++kt, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1)) { alive = false; break; }
          const uint32_t fb = mapa(smem_u32(&full[s]), 0);
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * Cfg::STAGE_BYTES);
          uint8_t* sa = smem + s * Cfg::STAGE_BYTES;
          tma_load_2d_pair(sa, &tmA, kt * GEMM_BK, wrow, fb);
          tma_load_2d_pair(sa + Cfg::A_BYTES, &tmB, kt * GEMM_BK, trow, fb);
        }
        if (!alive) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int it = 0, j = 0;
      bool alive = true;
      for (int w = pair; w < p.n_work && alive; w += n_pairs, ++j) {
        const Tile t = decode_pair_tile(p, w);
        const int acc = j & 1;
        if (!mbar_wait_cluster(&tempty[acc], ((j >> 1) & 1) ^ 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)acc * Cfg::ACC_STRIDE;
        for (int kt = t.kt0; kt < t.kt1; ++kt, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1)) { alive = false; break; }
          if (kt == t.kt0 && j < 3) trace_stamp(p, 2 + 4 * j);
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * Cfg::STAGE_BYTES);
          const uint64_t da = smem_desc_sw128(sa);
          const uint64_t db = smem_desc_sw128(sa + Cfg::A_BYTES);
#pragma unroll
          for (int kk = 0; kk < GEMM_BK / 16; ++kk)
            mma2_bf16(d_tmem, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), IDESC,
                      (kt > t.kt0 || kk > 0) ? 1u : 0u);
          commit2_both(&empty[s]);
        }
        if (alive) commit2_both(&tfull[acc]);
        if (j < 3) trace_stamp(p, 3 + 4 * j);
      }
    }
  } else {
    const int q = warp & 3;
    int j = 0, uses = 0;
    uint8_t* stg = smem + Cfg::OFF_STG + (warp - 2) * STG_WARP;
    const uint32_t te_leader[2] = {mapa(smem_u32(&tempty[0]), 0), mapa(smem_u32(&tempty[1]), 0)};
    for (int w = pair; w < p.n_work; w += n_pairs, ++j) {
      const Tile t = decode_pair_tile(p, w);
      const int acc = j & 1;
      const int f0 = (t.m0 << 1) + (int)rank * 128 + q * 32;  // the warp's weight rows
      const bool ok = mbar_wait(&tfull[acc], (j >> 1) & 1);
      __syncwarp();
      if (!ok) break;
      if (warp == 2 && lane == 0 && j < 3) trace_stamp(p, 4 + 4 * j);
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)acc * Cfg::ACC_STRIDE;
      epilogue_pair<BN, EPI>(p, &tmO, taddr, stg, f0, t.nt * BN, t.split, lane, uses);
      if (warp == 2 && lane == 0 && j < 3) trace_stamp(p, 5 + 4 * j);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(te_leader[acc]);
    }
    if (lane == 0) bulk_wait0();  // stores complete before the CTA exits
    __syncwarp();
  }
  tc_fence_before();
  cluster_sync_all();  // every MMA, commit and remote arrival is done
  if (threadIdx.x == 0) trace_stamp(p, 14);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem, Cfg::TMEM_COLS);
  }
}

}  // namespace pair
}  // namespace fvb
