// Persistent form of the contraction engine for the one-pass modes (TF32,
// bf16) on TMA-fed operands (dense A or dense-with-zeros upper A, dense B):
// C(M x N) = A(M x K) * B(K x N), 256 x 256 output tiles on CTA pairs
// (tcgen05.mma.cta_group::2), as in umma_gemm_kernel.
//
// One cluster (CTA pair) per SM pair walks the tiles t = cluster, cluster +
// clusters, ... in the grouped rasterisation order.  The stage ring runs on
// across tiles, and the accumulator is double-buffered in tensor memory
// (2 x 256 columns): while the epilogue warps read tile t out of one buffer
// and store it, the MMA issuer already accumulates tile t+1 into the other.
// Per-tile launch, tensor-memory allocation and barrier set-up are paid once
// per CTA instead of once per tile.
//
// Warp roles (224 threads):
//   warp 0      TMA producer (one lane): this CTA's 128 A rows and 128 B columns
//   warp 1      TMEM allocator + MMA issuer (one lane of the leader CTA)
//   warps 2-5   epilogue: warp w reads TMEM lanes 32 (w % 4).. (all 256
//               columns) and stores its rows of C
//   warp 6      relay (one lane): this CTA's TMA completion -> the leader's
//               `ready` barrier (the pair MMA reads both CTAs' stages)
//
// Barriers: full[s] (this CTA's TMA bytes), ready[s] (leader: one relay
// arrival per CTA), empty[s] (MMA commit, both CTAs), acc_full[b] (MMA
// commit of buffer b, both CTAs), acc_empty[b] (leader: one arrival per
// epilogue warp of both CTAs), mma_done (every MMA issued has completed).
// Every wait is bounded (WaitCtx); on expiry the roles stop, copies and MMAs
// in flight are drained, tensor memory is freed and the CTA exits.
#pragma once
#include "smm_umma.cuh"

namespace smm {

constexpr int kPersistThreads = 224;
constexpr int kPersistBN = 256;

template <AKind AK, Mode MD>
__host__ __device__ constexpr int persist_stage_bytes() {
  return umma_stage_bytes<AK, MD, kPersistBN / 2>();
}
template <AKind AK, Mode MD>
__host__ __device__ constexpr int persist_stages() {
  return umma_stages<AK, MD, kPersistBN / 2>();
}
template <AKind AK, Mode MD>
__host__ __device__ constexpr int persist_smem_bytes() {
  return 1024 + persist_stages<AK, MD>() * persist_stage_bytes<AK, MD>() + 512;
}

template <AKind AK, Mode MD>
__global__ void __launch_bounds__(kPersistThreads, 1)
    umma_persist_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const UmmaParams p) {
  static_assert(MD != Mode::TF32x3, "one-pass modes only");
  static_assert(AK == AKind::Dense || AK == AKind::UpperDense, "TMA-fed left operands only");
  using MT = ModeTraits<MD>;
  constexpr int BN = kPersistBN;
  constexpr int KS = MT::kStageK;
  constexpr int kBCols = BN / 2;
  constexpr int kBTile = TileGeom<kBCols>::kBTileBytes;
  constexpr int kSubs = umma_subs<AK, MD, kBCols>();
  constexpr int STAGES = persist_stages<AK, MD>();
  constexpr int kStage = persist_stage_bytes<AK, MD>();
  constexpr uint32_t kTxBytes = kSubs * (kATileBytes + kBTile);
  constexpr uint32_t kIdesc = make_idesc(MT::kFmt, 2 * kBM, BN, 0, 1);
  constexpr uint32_t kTmemCols = 2 * BN;  // two accumulator buffers
  constexpr uint32_t kEpiWarps = 4;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStage);
  uint64_t* ready = full + STAGES;
  uint64_t* empty = ready + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto a_t = [&](int s) { return smem + s * kStage; };
  auto b_t = [&](int s) { return smem + s * kStage + kSubs * kATileBytes; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  auto in_cta = [&](uint64_t* bar, uint32_t r) { return mapa_shared(smem_u32(bar), r); };

  const int cluster = static_cast<int>(blockIdx.x >> 1);
  const int clusters = static_cast<int>(gridDim.x >> 1);
  const int tiles = p.row_tiles * p.col_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 2);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, kTmemCols);
  tc_fence_before_sync();
  cluster_sync_all();  // both CTAs' barriers initialised before any remote arrival
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  const WaitCtx wprod{abort_flag, p.status, p.wait_limit_ns, kWaitProducer};
  const WaitCtx wmma{abort_flag, p.status, p.wait_limit_ns, kWaitMma};
  const WaitCtx wxf{abort_flag, p.status, p.wait_limit_ns, kWaitTransform};
  const WaitCtx wepi{abort_flag, p.status, p.wait_limit_ns, kWaitEpilogue};

  // Tile t -> its rows, columns and k-block range (grouped rasterisation;
  // for the triangular operand the K range starts at the tile's first row).
  auto tile_of = [&](int t, int& tile_m0, int& n0, int& kb_begin, int& num_kb) {
    const int per_group = p.raster_group * p.col_tiles;
    const int g = t / per_group;
    const int first = g * p.raster_group;
    const int rows_here = min(p.raster_group, p.row_tiles - first);
    const int in = t - g * per_group;
    tile_m0 = (first + in % rows_here) * 2 * kBM;
    n0 = (in / rows_here) * BN;
    kb_begin = 0;
    if constexpr (AK == AKind::UpperDense) kb_begin = a_struct_row(p, tile_m0) / KS;
    const int kb_end = (p.K + KS - 1) / KS;
    num_kb = (max(kb_end - kb_begin, 0) + kSubs - 1) / kSubs;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int g = 0;  // stages issued so far (all tiles)
      bool ok = true;
      for (int t = cluster; ok && t < tiles; t += clusters) {
        int tile_m0, n0, kb_begin, num_kb;
        tile_of(t, tile_m0, n0, kb_begin, num_kb);
        const int m0 = tile_m0 + static_cast<int>(rank) * kBM;
        const int nb0 = n0 + static_cast<int>(rank) * kBCols;
        for (int i = 0; i < num_kb; ++i, ++g) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, wprod)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], kTxBytes);
#pragma unroll
          for (int j = 0; j < kSubs; ++j) {
            const int k0 = (kb_begin + i * kSubs + j) * KS;
            tma_load_2d(a_t(s) + j * kATileBytes, &tmA, &full[s], k0, m0);
#pragma unroll
            for (int c = 0; c < kBCols / MT::kBoxCols; ++c)
              tma_load_2d(b_t(s) + j * kBTile + c * MT::kBoxBytes, &tmB, &full[s], nb0 + MT::kBoxCols * c, k0);
          }
        }
      }
      if (!ok || *abort_flag) {
        // no bulk copy may land after the CTA has exited (bounded drain)
        volatile int no_abort = 0;
        const WaitCtx drain{&no_abort, p.status, p.drain_limit_ns, kWaitDrain};
        for (int i = (g > STAGES ? g - STAGES : 0); i < g; ++i) mbar_wait(&full[i % STAGES], (i / STAGES) & 1, drain);
      }
    }
  } else if (warp == 6) {
    // ------------------------------------------------------------ relay
    if (lane == 0) {
      const uint32_t ready0 = in_cta(&ready[0], 0);
      int g = 0;
      bool ok = true;
      for (int t = cluster; ok && t < tiles; t += clusters) {
        int tile_m0, n0, kb_begin, num_kb;
        tile_of(t, tile_m0, n0, kb_begin, num_kb);
        for (int i = 0; i < num_kb; ++i, ++g) {
          const int s = g % STAGES;
          if (!mbar_wait(&full[s], (g / STAGES) & 1, wxf)) {
            ok = false;
            break;
          }
          fence_proxy_async_smem();
          mbar_arrive_cluster(ready0 + 8u * s);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      const uint64_t dA0 = make_smem_desc(smem_u32(a_t(0)), 16, 512, kLayoutSw64);
      const uint64_t dB0 = make_smem_desc(smem_u32(b_t(0)), MT::kBoxBytes, MT::kBSbo, MT::kBLayout);
      const uint32_t a_lo0 = static_cast<uint32_t>(dA0), a_hi32 = static_cast<uint32_t>(dA0 >> 32);
      const uint32_t b_lo0 = static_cast<uint32_t>(dB0), b_hi32 = static_cast<uint32_t>(dB0 >> 32);
      constexpr uint32_t kAKStep = 32 >> 4, kBKStep = MT::kBStepBytes >> 4;
      constexpr uint32_t kStageOff = kStage >> 4;
      const uint32_t ready_c = smem_u32(&ready[0]);
      const uint32_t empty_c[2] = {in_cta(&empty[0], 0), in_cta(&empty[0], 1)};
      const uint32_t accf_c[2][2] = {{in_cta(&acc_full[0], 0), in_cta(&acc_full[0], 1)},
                                     {in_cta(&acc_full[1], 0), in_cta(&acc_full[1], 1)}};
      int s = 0, lt = 0;
      uint32_t ph = 0, soff = 0;
      bool ok = true;
      for (int t = cluster; ok && t < tiles; t += clusters, ++lt) {
        int tile_m0, n0, kb_begin, num_kb;
        tile_of(t, tile_m0, n0, kb_begin, num_kb);
        const int buf = lt & 1;
        // the epilogue of the tile that last used this buffer has read it out
        if (!mbar_wait(&acc_empty[buf], ((lt >> 1) & 1) ^ 1, wmma)) break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        for (int i = 0; i < num_kb; ++i) {
          if (!mbar_try_wait(ready_c + 8u * s, ph) && !mbar_wait(&ready[s], ph, wmma)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
#pragma unroll
          for (int q = 0; q < 2 * kSubs; ++q) {
            const int j = q >> 1, kk = q & 1;
            const uint32_t al = a_lo0 + soff + j * (kATileBytes >> 4) + kk * kAKStep;
            const uint32_t bl = b_lo0 + soff + j * (kBTile >> 4) + kk * kBKStep;
            umma_lohi<true, MT::kBf16>(d_tmem, al, a_hi32, bl, b_hi32, kIdesc, (i > 0 || q > 0) ? 1u : 0u);
          }
          umma_commit_addr<true>(empty_c[0] + 8u * s);
          umma_commit_addr<true>(empty_c[1] + 8u * s);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
            soff = 0;
          } else {
            soff += kStageOff;
          }
        }
        if (!ok) break;
        // buffer `buf` holds tile t once every MMA issued so far has completed
        umma_commit_addr<true>(accf_c[buf][0]);
        umma_commit_addr<true>(accf_c[buf][1]);
      }
      // tensor memory quiescent before it is freed (bounded, ignoring the abort flag)
      umma_commit_addr<true>(in_cta(mma_done, 0));
      volatile int no_abort = 0;
      const WaitCtx drain{&no_abort, p.status, p.drain_limit_ns, kWaitDrain};
      mbar_wait(mma_done, 0, drain);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5)
    const int q = warp & 3;  // TMEM lanes 32q.. of this CTA's accumulator rows
    const uint32_t acc_empty0 = in_cta(&acc_empty[0], 0);
    const bool vec = (p.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
    int lt = 0;
    for (int t = cluster; t < tiles; t += clusters, ++lt) {
      int tile_m0, n0, kb_begin, num_kb;
      tile_of(t, tile_m0, n0, kb_begin, num_kb);
      const int buf = lt & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (lt >> 1) & 1, wepi))) break;
      tc_fence_after_sync();
      const int row = tile_m0 + static_cast<int>(rank) * kBM + q * 32 + lane;
      float* crow = p.C + static_cast<long long>(row) * p.ldc;
      const uint32_t col0 = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        if (num_kb > 0) {
          tmem_ld_32x32b_x16(col0 + c, *reinterpret_cast<uint32_t(*)[16]>(r));
          tmem_ld_32x32b_x16(col0 + c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = 0u;
        }
        const int col = n0 + c;
        if (row < p.M) {
          if (vec && col + 32 <= p.N) {
            float4* dst = reinterpret_cast<float4*>(crow + col);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                   __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
          } else {
#pragma unroll
            for (int v = 0; v < 32; ++v)
              if (col + v < p.N) crow[col + v] = __uint_as_float(r[v]);
          }
        }
      }
      // buffer read out: the MMA may overwrite it
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0 + 8u * buf);
    }
  }

  tc_fence_before_sync();
  // Neither CTA leaves while the leader's MMAs may still read the other's
  // shared memory or the other may still arrive on the leader's barriers.
  cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace smm
