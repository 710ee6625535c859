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
//          weight rows), then a release-arrive on the leader's tempty[]
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

template <int BN>
struct PairCfg {
  static_assert(BN % 16 == 0 && (BN / 2) % 8 == 0 && BN >= 64 && BN <= 256, "block_n");
  static constexpr int A_BYTES = 128 * GEMM_BK * 2;
  static constexpr int B_BYTES = (BN / 2) * GEMM_BK * 2;  // this CTA's half
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES < 8 ? (200 * 1024) / STAGE_BYTES : 8;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 256 ? 256u : 512u;
  static constexpr uint32_t ACC_STRIDE = TMEM_COLS / 2;  // accumulator columns
};

// Work item w of the pairs: weight row pair tile (256 rows) fastest, then
// token tile, then K split (same decode as the one-SM kernel with
// m_tiles counting 256-row pair tiles).
template <int BN, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, const GemmDev p) {
  using Cfg = PairCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = idesc_bf16_f32(256, BN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2]
  uint64_t* tempty = tfull + 2;      // [2] (leader: 4 warps x 2 CTAs)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;

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
  }
  if (warp == 1) tmem_alloc2(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int w = pair; w < p.n_work; w += n_pairs) {
        const Tile t = decode_tile(p, w);
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
        const Tile t = decode_tile(p, w);
        const int acc = j & 1;
        if (!mbar_wait_cluster(&tempty[acc], ((j >> 1) & 1) ^ 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)acc * Cfg::ACC_STRIDE;
        for (int kt = t.kt0; kt < t.kt1; ++kt, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1)) { alive = false; break; }
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
      }
    }
  } else {
    const int q = warp & 3;
    int j = 0;
    const uint32_t te_leader[2] = {mapa(smem_u32(&tempty[0]), 0), mapa(smem_u32(&tempty[1]), 0)};
    for (int w = pair; w < p.n_work; w += n_pairs, ++j) {
      const Tile t = decode_tile(p, w);
      const int acc = j & 1;
      const int f = (t.m0 << 1) + (int)rank * 128 + q * 32 + lane;  // weight row
      EpiPre pre;
      epi_prefetch<BN, EPI, true>(p, pre, nullptr, f, t.nt * BN, t.split, lane);
      const bool ok = mbar_wait(&tfull[acc], (j >> 1) & 1);
      __syncwarp();
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)acc * Cfg::ACC_STRIDE;
      epilogue_swap<BN, EPI, FVB_ACT_NONE, false>(p, pre, taddr, nullptr, f, t.nt * BN, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(te_leader[acc]);
    }
  }
  tc_fence_before();
  cluster_sync_all();  // every MMA, commit and remote arrival is done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem, Cfg::TMEM_COLS);
  }
}

}  // namespace pair
}  // namespace fvb
