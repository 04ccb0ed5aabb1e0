// matmul.cu -- C[M,N] = A[M,K] . B[K,N] on the sm_100a tensor cores.
//
// The reference family (matmul_gen.cpp:287-402) stages fp32 copies of the
// tiles in shared memory and accumulates with scalar FMAs.  Here:
//
//   * persistent kernel, one CTA per SM, tiles of 128 x BN (BN 64/128/256)
//     or, config tile_m 256 with cta_group 1, 256 x BN: two M=128 MMAs per
//     K-step share each B tile, so a third less operand traffic reaches the
//     SM per FLOP at BN 256 (TMEM: two accumulator halves of BN columns),
//     raster grouped by `group_m` M-tiles for L2 reuse (or, group_m < 0,
//     banded by N-tiles with the band's B panels kept in L2);
//   * warp 0 (one lane) is the TMA producer: per K-block of 64 it loads the
//     A box [128 rows x 64 K] and BN/64 B boxes [64 K x 64 N], all with the
//     128-byte swizzle, into a STAGES-deep shared-memory ring (full/empty
//     mbarriers);
//   * warp 1 (one lane) issues tcgen05.mma kind::f16 (bf16 x bf16 -> fp32),
//     M=128, N=BN, K=16, four per K-block, A K-major and B MN-major straight
//     from the swizzled tiles (no transpose pass), accumulating in TMEM;
//     tcgen05.commit releases each ring slot and, per tile, signals the
//     epilogue; warp 1 also owns the TMEM allocation;
//   * warps 2-5 are the epilogue: each reads its 32-lane quadrant of the
//     fp32 accumulator with tcgen05.ld, rounds to bf16 once and stores the
//     tile with TMA through swizzled shared-memory staging; ACC TMEM buffers
//     let the next tile's MMAs run meanwhile, and with 256-row tiles each
//     128-row half is freed as soon as it is drained, so the next tile's
//     half-0 MMAs overlap the drain of half 1.
//
// Every mbarrier wait is bounded (KsWait): on timeout the kernel records the
// error word, waits (bounded) for its own TMA loads and MMAs, frees TMEM and
// returns.  No multicast loads anywhere.
#include <atomic>
#include <cmath>

#include "ks_common.cuh"

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;                    // one 128-byte swizzle row of bf16
constexpr int kUmmaK = 16;
constexpr int kThreads = 192;              // 6 warps: producer, MMA, 4 x epilogue
constexpr uint32_t kABytes = kBM * kBK * 2;  // 16 KB per stage
constexpr uint32_t kBBoxBytes = kBK * 64 * 2;  // one B box: 64 K-rows x 64 N-cols = 8 KB

// Epilogue staging for the TMA store of C: per epilogue warp two buffers of
// [32 rows x 32 columns] bf16 (64-byte rows, 64-byte swizzle), 2 KB each.
constexpr uint32_t kCBuf = 32 * 64;
constexpr uint32_t kCStage = 4 * 2 * kCBuf;  // 4 warps x 2 buffers = 16 KB

template <int BN, int STAGES, int ACC, int MH = 1>
struct MmLayout {
  static constexpr uint32_t a_bytes = MH * kABytes;  // MH 128-row A boxes per stage
  static constexpr uint32_t b_bytes = kBK * BN * 2;
  static constexpr uint32_t a_off = 0;
  static constexpr uint32_t b_off = a_off + STAGES * a_bytes;
  static constexpr uint32_t c_off = b_off + STAGES * b_bytes;  // 1024-aligned (stage sizes are multiples of 8 KB)
  static constexpr uint32_t bar_off = c_off + kCStage;
  // full[STAGES], empty[STAGES], tfull[ACC], tempty[ACC * MH] (one per 128-row half), drain
  static constexpr uint32_t n_bars = 2 * STAGES + ACC + ACC * MH + 1;
  static constexpr uint32_t misc_off = bar_off + n_bars * 8;
  static constexpr uint32_t bytes = misc_off + 16;
  static constexpr uint32_t smem_request = bytes + 1024;  // slack to align the base to 1024
  static constexpr uint32_t tmem_cols_raw = ACC * BN * MH;
  static constexpr uint32_t tmem_cols = tmem_cols_raw <= 32 ? 32 : tmem_cols_raw <= 64 ? 64
                                        : tmem_cols_raw <= 128 ? 128 : tmem_cols_raw <= 256 ? 256 : 512;
  static_assert(tmem_cols_raw <= 512, "TMEM holds 512 columns");
};

// Output tile t of the persistent raster.  group_m > 0: groups of group_m
// M-tiles, M-tiles fastest, so the A panels of a group are reused while B
// streams past.  group_m < 0: bands of -group_m N-tiles, N-tiles fastest, so
// the band's B panels (loaded with evict_last) stay in L2 while all of A
// streams past once per band; for tall problems (M >> N) this reads less.
KS_DEV void tile_coords(int t, int num_m, int num_n, int group_m, int &tm, int &tn) {
  if (group_m < 0) {
    const int band_n = -group_m;
    const int band_size = band_n * num_m;
    const int b = t / band_size;
    const int first_n = b * band_n;
    const int bn = min(num_n - first_n, band_n);
    const int r = t - b * band_size;
    tn = first_n + r % bn;
    tm = r / bn;
    return;
  }
  const int group_size = group_m * num_n;
  const int g = t / group_size;
  const int first_m = g * group_m;
  const int gm = min(num_m - first_m, group_m);
  const int r = t - g * group_size;
  tm = first_m + r % gm;
  tn = r / gm;
}

template <int BN, int STAGES, int ACC, int MH = 1>
__global__ void __launch_bounds__(kThreads, 1)
    matmul_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap tma_c, int M, int N, int K, int group_m, int b3d,
                     KsWait wait) {
  using L = MmLayout<BN, STAGES, ACC, MH>;
  constexpr int kTM = kBM * MH;  // output tile rows: MH M=128 MMAs share each B tile
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ks_smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::bar_off);
  uint64_t *full = bars;
  uint64_t *empty = bars + STAGES;
  uint64_t *tfull = bars + 2 * STAGES;
  uint64_t *tempty = bars + 2 * STAGES + ACC;  // [acc * MH + half]
  uint64_t *drain = bars + 2 * STAGES + ACC + ACC * MH;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::misc_off);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + L::misc_off + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + kTM - 1) / kTM, num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ks_mbar_init(full + s, 1);
      ks_mbar_init(empty + s, 1);
    }
    for (int a = 0; a < ACC; ++a) ks_mbar_init(tfull + a, 1);
    for (int a = 0; a < ACC * MH; ++a) ks_mbar_init(tempty + a, 4);
    ks_mbar_init(drain, 1);
    *abort = 0;
    ks_fence_mbar_init();
    ks_prefetch_tmap(&tma_a);
    ks_prefetch_tmap(&tma_b);
    ks_prefetch_tmap(&tma_c);
  }
  if (warp == 1) {
    ks_tmem_alloc(tmem_slot, L::tmem_cols);
    ks_tmem_relinquish();
  }
  ks_tc_fence_before();
  __syncthreads();
  ks_tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t armed = 0, armed_parity = 0;  // per-stage bits for the teardown wait
    bool ok = true;
    const bool keep_b = group_m < 0;  // N-band raster: the band's B panels stay in L2
    const uint64_t pol = ks_l2_policy_evict_last();
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
      int tm, tn;
      tile_coords(t, num_m, num_n, group_m, tm, tn);
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!ks_mbar_wait(empty + stage, phase ^ 1u, abort, wait)) {
          ok = false;
          break;
        }
        uint8_t *a_dst = smem + L::a_off + stage * L::a_bytes;
        uint8_t *b_dst = smem + L::b_off + stage * L::b_bytes;
        ks_mbar_arrive_expect_tx(full + stage, L::a_bytes + L::b_bytes);
#pragma unroll
        for (int h = 0; h < MH; ++h) ks_tma_load_2d(a_dst + h * kABytes, &tma_a, full + stage, kb * kBK, tm * kTM + h * kBM);
        if (b3d) {
          // one copy for all BN/64 column blocks (tensor map dims: 64 columns, K, N/64)
          if (keep_b)
            ks_tma_load_3d_hint(b_dst, &tma_b, full + stage, 0, kb * kBK, tn * (BN / 64), pol);
          else
            ks_tma_load_3d(b_dst, &tma_b, full + stage, 0, kb * kBK, tn * (BN / 64));
        } else {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) {
            if (keep_b)
              ks_tma_load_2d_hint(b_dst + j * kBBoxBytes, &tma_b, full + stage, tn * BN + j * 64, kb * kBK, pol);
            else
              ks_tma_load_2d(b_dst + j * kBBoxBytes, &tma_b, full + stage, tn * BN + j * 64, kb * kBK);
          }
        }
        armed |= 1u << stage;
        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // teardown: every load this thread issued must have landed before exit
    for (int s = 0; s < STAGES; ++s)
      if (armed & (1u << s)) ks_mbar_wait(full + s, (armed_parity >> s) & 1u, nullptr, wait);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = ks_idesc_bf16_f32(kBM, BN, false, true);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int i = 0;
    // MMAs of K-block kb for the 128-row halves [h0, h1) of the tile, from ring stage st
    auto issue = [&](int st, int kb, uint32_t d_tmem, int h0, int h1) {
      const uint32_t a_addr = ks_smem_u32(smem + L::a_off + st * L::a_bytes);
      const uint32_t b_addr = ks_smem_u32(smem + L::b_off + st * L::b_bytes);
#pragma unroll
      for (int k = 0; k < kBK / kUmmaK; ++k) {
        // B: MN-major, 64-column boxes kBBoxBytes apart (LBO), 8 K-rows 1024 bytes apart (SBO);
        // step 16 K-rows = 2048 bytes per K=16.
        const uint64_t bdesc = ks_umma_desc_sw128(b_addr + k * 2048, kBBoxBytes, 1024);
#pragma unroll
        for (int h = 0; h < MH; ++h) {
          if (h < h0 || h >= h1) continue;
          // A: K-major, 128-byte rows, 8-row groups 1024 bytes apart; step 32 bytes per K=16.
          const uint64_t adesc = ks_umma_desc_sw128(a_addr + h * kABytes + k * 32, 16, 1024);
          ks_umma_ss(d_tmem + h * BN, adesc, bdesc, idesc, (kb | k) != 0);
        }
      }
    };
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++i) {
      const int acc = i % ACC;
      const uint32_t acc_phase = (i / ACC) & 1;
      // The epilogue frees the accumulator one 128-row half at a time.  Half
      // 0's MMAs start as soon as it is free; those of the other halves wait
      // for theirs, deferred over at most STAGES - 1 K-blocks (their ring
      // stages are released once they are issued), so the tensor core works
      // on half 0 while the epilogue still drains the rest.
      if (!ks_mbar_wait(tempty + acc * MH, acc_phase ^ 1u, abort, wait)) break;
      ks_tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN * MH;
      bool rest_free = MH == 1;
      int pend = 0;  // K-blocks before kb whose other-half MMAs are deferred
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!ks_mbar_wait(full + stage, phase, abort, wait)) {
          ok = false;
          break;
        }
        ks_tc_fence_after();
        issue(stage, kb, d_tmem, 0, 1);
        if (!rest_free) {
          if (pend + 1 < STAGES && kb + 1 < num_kb &&
              !ks_mbar_test_wait(ks_smem_u32(tempty + acc * MH + 1), acc_phase ^ 1u)) {
            ++pend;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          for (int h = 1; h < MH && ok; ++h) ok = ks_mbar_wait(tempty + acc * MH + h, acc_phase ^ 1u, abort, wait);
          if (!ok) break;
          ks_tc_fence_after();
          rest_free = true;
          for (int p = pend; p > 0; --p) {
            const int sp = (stage + STAGES - p) % STAGES;
            issue(sp, kb - p, d_tmem, 1, MH);
            ks_umma_commit(empty + sp);
          }
          pend = 0;
        }
        issue(stage, kb, d_tmem, 1, MH);
        ks_umma_commit(empty + stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) ks_umma_commit(tfull + acc);
    }
    // teardown: all MMAs issued by this thread complete before TMEM is freed
    ks_umma_commit(drain);
    ks_mbar_wait(drain, 0, nullptr, wait);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    // Each warp drains its 32 accumulator lanes (rows) 32 columns at a time:
    // tcgen05.ld, round to bf16, write the [32 x 32] block into one of its two
    // swizzled staging buffers, and lane 0 stores the block with TMA (the
    // store clips rows >= M and columns >= N).  The accumulator is released
    // as soon as its last columns are in registers.
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    uint8_t *stg = smem + L::c_off + (warp - 2) * 2 * kCBuf;
    int i = 0;
    uint32_t nstore = 0;  // blocks this warp has stored (buffer = nstore & 1)
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++i) {
      const int acc = i % ACC;
      const uint32_t acc_phase = (i / ACC) & 1;
      if (!ks_mbar_wait(tfull + acc, acc_phase, abort, wait)) break;
      ks_tc_fence_after();
      int tm, tn;
      tile_coords(t, num_m, num_n, group_m, tm, tn);
      const uint32_t t_addr = tmem_base + (uint32_t(q * 32) << 16) + acc * BN * MH;
#pragma unroll 1
      for (int cc = 0; cc < MH * (BN / 32); ++cc) {
        const int h = cc / (BN / 32);  // 128-row half of the tile
        uint32_t r[32];
        ks_tmem_ld32(t_addr + cc * 32, r);
        ks_tmem_wait_ld();
        if ((cc + 1) % (BN / 32) == 0) {  // this half is free for the next tile's MMAs
          ks_tc_fence_before();
          __syncwarp();
          if (lane == 0) ks_mbar_arrive(tempty + acc * MH + h);
        }
        if (num_kb == 0) continue;  // K = 0 is written by the host (zeros)
        uint8_t *buf = stg + (nstore & 1) * kCBuf;
        if (lane == 0) ks_bulk_wait_read<1>();  // the store two blocks back has read this buffer
        __syncwarp();
        // row = lane: four 16-byte chunks, chunk v at position v ^ ((lane >> 1) & 3) (64-byte swizzle)
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          w.x = ks_pack_bf16x2(__uint_as_float(r[v * 8 + 0]), __uint_as_float(r[v * 8 + 1]));
          w.y = ks_pack_bf16x2(__uint_as_float(r[v * 8 + 2]), __uint_as_float(r[v * 8 + 3]));
          w.z = ks_pack_bf16x2(__uint_as_float(r[v * 8 + 4]), __uint_as_float(r[v * 8 + 5]));
          w.w = ks_pack_bf16x2(__uint_as_float(r[v * 8 + 6]), __uint_as_float(r[v * 8 + 7]));
          *reinterpret_cast<uint4 *>(buf + lane * 64 + ((v ^ ((lane >> 1) & 3)) * 16)) = w;
        }
        ks_fence_proxy_async();  // the generic-proxy writes are visible to the TMA store
        __syncwarp();
        if (lane == 0) {
          ks_tma_store_2d(&tma_c, buf, tn * BN + (cc % (BN / 32)) * 32, tm * kTM + h * kBM + q * 32);
          ks_bulk_commit_group();
        }
        ++nstore;
      }
    }
    if (lane == 0) ks_bulk_wait_all();  // C is in global memory before the CTA exits
  }

  ks_tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ks_tc_fence_after();
    ks_tmem_dealloc(tmem_base, L::tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// Pair kernel (config tile_m 256): clusters of two CTAs on two SMs compute
// 256 x BN output tiles with tcgen05 cta_group::2 MMAs (M=256).  Each CTA
// loads its own 128 rows of A and half (BN/2 columns) of B per K-block, so an
// SM streams 16 KB of A and BN/2 * 128 bytes of B per 128 x BN x 64 step
// instead of 16 KB + BN * 128 bytes: B traffic from L2 halves.
//
//   * warp 0 (both CTAs): TMA producer for its own shared memory; the
//     completion bytes of both CTAs' loads count on the even CTA's `full`
//     barrier (the even producer expects both halves);
//   * warp 1 (even CTA): issues the pair MMAs; each stage's commit arrives
//     on `empty` in both CTAs, each tile's on `tfull` in both CTAs;
//   * warps 2-5 (both CTAs): epilogue of the CTA's 128 accumulator lanes (its
//     128 rows of the tile, all BN columns), then arrive on the even CTA's
//     `tempty` (8 warps per tile).
//
// All waits are bounded.  Both CTAs stay resident until the pair is done
// (cluster barriers at start and end): the even CTA's MMAs read the odd
// CTA's shared memory and write its TMEM.  No load uses multicast.
// ---------------------------------------------------------------------------
template <int BN, int STAGES, int ACC>
struct Mm2Layout {
  static constexpr uint32_t b_bytes = kBK * (BN / 2) * 2;  // this CTA's half of a B stage
  static constexpr uint32_t a_off = 0;
  static constexpr uint32_t b_off = a_off + STAGES * kABytes;
  static constexpr uint32_t c_off = b_off + STAGES * b_bytes;  // C staging, 1024-aligned
  static constexpr uint32_t bar_off = c_off + kCStage;
  // full[STAGES], empty[STAGES], tfull[ACC], tempty[ACC], drain
  static constexpr uint32_t n_bars = 2 * STAGES + 2 * ACC + 1;
  static constexpr uint32_t misc_off = bar_off + n_bars * 8;
  static constexpr uint32_t bytes = misc_off + 16;
  static constexpr uint32_t smem_request = bytes + 1024;
  static constexpr uint32_t tmem_cols_raw = ACC * BN;
  static constexpr uint32_t tmem_cols = tmem_cols_raw <= 32 ? 32 : tmem_cols_raw <= 64 ? 64
                                        : tmem_cols_raw <= 128 ? 128 : tmem_cols_raw <= 256 ? 256 : 512;
};

template <int BN, int STAGES, int ACC>
__global__ void __launch_bounds__(kThreads, 1)
    matmul_tc2_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                      const __grid_constant__ CUtensorMap tma_c, int M, int N, int K, int group_m, KsWait wait) {
  using L = Mm2Layout<BN, STAGES, ACC>;
  constexpr int kPM = 2 * kBM;  // rows per pair tile
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ks_smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::bar_off);
  uint64_t *full = bars;
  uint64_t *empty = bars + STAGES;
  uint64_t *tfull = bars + 2 * STAGES;
  uint64_t *tempty = bars + 2 * STAGES + ACC;
  uint64_t *drain = bars + 2 * STAGES + 2 * ACC;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::misc_off);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + L::misc_off + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = ks_cluster_ctarank();  // 0: issues the MMAs
  const int pair = int(blockIdx.x >> 1), num_pairs = int(gridDim.x >> 1);
  const int num_m = (M + kPM - 1) / kPM, num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ks_mbar_init(full + s, 1);
      ks_mbar_init(empty + s, 1);
    }
    for (int a = 0; a < ACC; ++a) {
      ks_mbar_init(tfull + a, 1);
      ks_mbar_init(tempty + a, 8);
    }
    ks_mbar_init(drain, 1);
    *abort = 0;
    ks_fence_mbar_init();
    ks_prefetch_tmap(&tma_a);
    ks_prefetch_tmap(&tma_b);
  }
  if (warp == 1) {
    ks_tmem_alloc_pair(tmem_slot, L::tmem_cols);
    ks_tmem_relinquish_pair();
  }
  ks_tc_fence_before();
  ks_cluster_sync();  // both CTAs' barriers are initialised before any remote signal
  ks_tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    const uint32_t full_even = ks_mapa(ks_smem_u32(full), 0);
    int stage = 0;
    uint32_t phase = 0;
    uint32_t armed = 0, armed_parity = 0;
    bool ok = true;
    for (int t = pair; t < num_tiles && ok; t += num_pairs) {
      int tm, tn;
      tile_coords(t, num_m, num_n, group_m, tm, tn);
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!ks_mbar_wait_cluster(empty + stage, phase ^ 1u, abort, wait)) {
          ok = false;
          break;
        }
        if (rank == 0) ks_mbar_arrive_expect_tx(full + stage, 2 * (kABytes + L::b_bytes));
        const uint32_t bar = full_even + stage * 8;
        uint8_t *a_dst = smem + L::a_off + stage * kABytes;
        uint8_t *b_dst = smem + L::b_off + stage * L::b_bytes;
        ks_tma_load_2d_pair(a_dst, &tma_a, bar, kb * kBK, tm * kPM + int(rank) * kBM);
#pragma unroll
        for (int j = 0; j < BN / 128; ++j)
          ks_tma_load_2d_pair(b_dst + j * kBBoxBytes, &tma_b, bar, tn * BN + int(rank) * (BN / 2) + j * 64,
                              kb * kBK);
        armed |= 1u << stage;
        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // teardown: every load issued here has landed (the even CTA's `full`
    // counts both CTAs' loads; a stage released on `empty` was consumed)
    for (int s = 0; s < STAGES; ++s)
      if (armed & (1u << s)) {
        if (rank == 0)
          ks_mbar_wait_cluster(full + s, (armed_parity >> s) & 1u, nullptr, wait);
        else
          ks_mbar_wait_cluster(empty + s, (armed_parity >> s) & 1u, nullptr, wait);
      }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = ks_idesc_bf16_f32(kPM, BN, false, true);
    const uint32_t empty_mine = ks_smem_u32(empty), empty_odd = ks_mapa(empty_mine, 1);
    const uint32_t tfull_mine = ks_smem_u32(tfull), tfull_odd = ks_mapa(tfull_mine, 1);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int i = 0;
    for (int t = pair; t < num_tiles && ok; t += num_pairs, ++i) {
      const int acc = i % ACC;
      const uint32_t acc_phase = (i / ACC) & 1;
      if (!ks_mbar_wait_cluster(tempty + acc, acc_phase ^ 1u, abort, wait)) break;
      ks_tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!ks_mbar_wait_cluster(full + stage, phase, abort, wait)) {
          ok = false;
          break;
        }
        ks_tc_fence_after();
        const uint32_t a_addr = ks_smem_u32(smem + L::a_off + stage * kABytes);
        const uint32_t b_addr = ks_smem_u32(smem + L::b_off + stage * L::b_bytes);
#pragma unroll
        for (int k = 0; k < kBK / kUmmaK; ++k) {
          // same descriptors as the single-CTA kernel; the hardware reads the
          // odd CTA's A rows and B columns at the same offsets
          const uint64_t adesc = ks_umma_desc_sw128(a_addr + k * 32, 16, 1024);
          const uint64_t bdesc = ks_umma_desc_sw128(b_addr + k * 2048, kBBoxBytes, 1024);
          ks_umma_ss_pair(d_tmem, adesc, bdesc, idesc, (kb | k) != 0);
        }
        ks_umma_commit_pair(empty_mine + stage * 8);
        ks_umma_commit_pair(empty_odd + stage * 8);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) {
        ks_umma_commit_pair(tfull_mine + acc * 8);
        ks_umma_commit_pair(tfull_odd + acc * 8);
      }
    }
    // teardown: all pair MMAs issued here complete before TMEM is freed
    ks_umma_commit_pair(ks_smem_u32(drain));
    ks_mbar_wait(drain, 0, nullptr, wait);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    // Same TMA-store epilogue as the one-CTA kernel, over this CTA's 128
    // rows of the 256-row pair tile.
    const uint32_t tempty_even = ks_mapa(ks_smem_u32(tempty), 0);
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    uint8_t *stg = smem + L::c_off + (warp - 2) * 2 * kCBuf;
    int i = 0;
    uint32_t nstore = 0;  // blocks this warp has stored (buffer = nstore & 1)
    for (int t = pair; t < num_tiles; t += num_pairs, ++i) {
      const int acc = i % ACC;
      const uint32_t acc_phase = (i / ACC) & 1;
      if (!ks_mbar_wait_cluster(tfull + acc, acc_phase, abort, wait)) break;
      ks_tc_fence_after();
      int tm, tn;
      tile_coords(t, num_m, num_n, group_m, tm, tn);
      const uint32_t t_addr = tmem_base + (uint32_t(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        uint32_t r[32];
        ks_tmem_ld32(t_addr + cc * 32, r);
        ks_tmem_wait_ld();
        if (cc + 1 == BN / 32) {  // the accumulator is free for the pair's next MMAs
          ks_tc_fence_before();
          __syncwarp();
          if (lane == 0) ks_mbar_arrive_cluster(tempty_even + acc * 8);
        }
        uint8_t *buf = stg + (nstore & 1) * kCBuf;
        if (lane == 0) ks_bulk_wait_read<1>();  // the store two blocks back has read this buffer
        __syncwarp();
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          w.x = ks_pack_bf16x2(__uint_as_float(r[v * 8 + 0]), __uint_as_float(r[v * 8 + 1]));
          w.y = ks_pack_bf16x2(__uint_as_float(r[v * 8 + 2]), __uint_as_float(r[v * 8 + 3]));
          w.z = ks_pack_bf16x2(__uint_as_float(r[v * 8 + 4]), __uint_as_float(r[v * 8 + 5]));
          w.w = ks_pack_bf16x2(__uint_as_float(r[v * 8 + 6]), __uint_as_float(r[v * 8 + 7]));
          *reinterpret_cast<uint4 *>(buf + lane * 64 + ((v ^ ((lane >> 1) & 3)) * 16)) = w;
        }
        ks_fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          ks_tma_store_2d(&tma_c, buf, tn * BN + cc * 32, tm * kPM + int(rank) * kBM + q * 32);
          ks_bulk_commit_group();
        }
        ++nstore;
      }
    }
    if (lane == 0) ks_bulk_wait_all();  // C is in global memory before the CTA exits
  }

  ks_tc_fence_before();
  __syncwarp();
  ks_cluster_sync();  // the pair's MMAs, loads and remote arrivals are done
  if (warp == 1) {
    ks_tc_fence_after();
    ks_tmem_dealloc_pair(tmem_base, L::tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// CUDA-core path for shapes the TMA path cannot take (K or N not a multiple
// of 8, or operands not 16-byte aligned): 64x64 output tile per CTA,
// 16 x 16 threads with a 4 x 4 register fragment, fp32 accumulate.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) matmul_simt_kernel(const uint16_t *__restrict__ a,
                                                          const uint16_t *__restrict__ b,
                                                          uint16_t *__restrict__ c, int M, int N, int K) {
  __shared__ float as[16][64 + 1];
  __shared__ float bs[16][64 + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int mm = i / 16, kk = i % 16;
      const int gm = m0 + mm, gk = k0 + kk;
      as[kk][mm] = (gm < M && gk < K) ? ks_bf16_to_f32(a[int64_t(gm) * K + gk]) : 0.f;
      const int kb = i / 64, nn = i % 64;
      const int gn = n0 + nn, gkb = k0 + kb;
      bs[kb][nn] = (gn < N && gkb < K) ? ks_bf16_to_f32(b[int64_t(gkb) * N + gn]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        av[u] = as[kk][ty + 16 * u];
        bv[u] = bs[kk][tx + 16 * u];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(av[u], bv[v], acc[u][v]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int gm = m0 + ty + 16 * u, gn = n0 + tx + 16 * v;
      if (gm < M && gn < N) c[int64_t(gm) * N + gn] = ks_f32_to_bf16(acc[u][v]);
    }
}

bool tc_shape_ok(const ks_matmul_args &a) {
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return a.k % 8 == 0 && a.n % 8 == 0 && al(a.a) && al(a.b) && al(a.out) && a.m < (1LL << 31) &&
         a.n < (1LL << 31) && a.k < (1LL << 31);
}

template <int BN, int STAGES, int ACC, int MH = 1>
int launch_tc(const ks_matmul_config &cfg, const ks_matmul_args &a, cudaStream_t st) {
  using L = MmLayout<BN, STAGES, ACC, MH>;
  CUtensorMap ta, tb;
  int s = ks::encode_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.a, uint64_t(a.k), uint64_t(a.m),
                             uint64_t(a.k) * 2, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (s != KS_OK) return s;
  // B as (64 columns, K, N/64 column blocks) when N is a multiple of 64, so
  // one copy per stage fetches all BN/64 blocks; else one 2-D box per block.
  int b3d = 0;
  if (BN > 64 && a.n % 64 == 0 &&
      ks::encode_tmap_3d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.b, 64, uint64_t(a.k), uint64_t(a.n / 64),
                         uint64_t(a.n) * 2, 128, 64, kBK, BN / 64, CU_TENSOR_MAP_SWIZZLE_128B) == KS_OK)
    b3d = 1;
  if (!b3d) {
    s = ks::encode_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.b, uint64_t(a.n), uint64_t(a.k),
                           uint64_t(a.n) * 2, 64, kBK, CU_TENSOR_MAP_SWIZZLE_128B);
    if (s != KS_OK) return s;
  }
  // C: [32 columns x 32 rows] boxes, 64-byte swizzle (the epilogue's staging layout)
  CUtensorMap tc;
  s = ks::encode_tmap_2d(&tc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.out, uint64_t(a.n), uint64_t(a.m),
                         uint64_t(a.n) * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  if (s != KS_OK) return s;
  auto kern = matmul_tc_kernel<BN, STAGES, ACC, MH>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(L::smem_request));
  if (e != cudaSuccess) return ks::map_cuda(e);
  const int64_t tiles = ((a.m + kBM * MH - 1) / (kBM * MH)) * ((a.n + BN - 1) / BN);
  const int sms = ks::sm_count();
  const int grid = int(tiles < sms ? tiles : sms);
  kern<<<grid, kThreads, L::smem_request, st>>>(ta, tb, tc, int(a.m), int(a.n), int(a.k), cfg.group_m, b3d,
                                                ks::wait_ctx());
  return ks::map_cuda(cudaGetLastError());
}

// Pair kernel launch: clusters of 2 via cudaLaunchKernelEx; the grid is the
// number of pairs that can be resident at once (cudaOccupancyMaxActiveClusters,
// queried once per device and instantiation), capped by the tile count.
template <int BN, int STAGES, int ACC>
int launch_tc2(const ks_matmul_config &cfg, const ks_matmul_args &a, cudaStream_t st) {
  using L = Mm2Layout<BN, STAGES, ACC>;
  CUtensorMap ta, tb;
  int s = ks::encode_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.a, uint64_t(a.k), uint64_t(a.m),
                             uint64_t(a.k) * 2, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (s != KS_OK) return s;
  s = ks::encode_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.b, uint64_t(a.n), uint64_t(a.k),
                         uint64_t(a.n) * 2, 64, kBK, CU_TENSOR_MAP_SWIZZLE_128B);
  if (s != KS_OK) return s;
  CUtensorMap tc;  // [32 columns x 32 rows] boxes, 64-byte swizzle (the epilogue's staging layout)
  s = ks::encode_tmap_2d(&tc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.out, uint64_t(a.n), uint64_t(a.m),
                         uint64_t(a.n) * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  if (s != KS_OK) return s;
  auto kern = matmul_tc2_kernel<BN, STAGES, ACC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(L::smem_request));
  if (e != cudaSuccess) return ks::map_cuda(e);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t lc = {};
  lc.blockDim = dim3(kThreads);
  lc.dynamicSmemBytes = L::smem_request;
  lc.stream = st;
  lc.attrs = attr;
  lc.numAttrs = 1;
  static std::atomic<int> max_pairs[64];  // per device; 0 = not queried yet
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return ks::map_cuda(e);
  int pairs_max = dev < 64 ? max_pairs[dev].load(std::memory_order_relaxed) : 0;
  if (pairs_max <= 0) {
    lc.gridDim = dim3(2 * unsigned(ks::sm_count() / 2));
    if ((e = cudaOccupancyMaxActiveClusters(&pairs_max, kern, &lc)) != cudaSuccess) return ks::map_cuda(e);
    if (pairs_max <= 0) return KS_ERR_LAUNCH;
    if (dev < 64) max_pairs[dev].store(pairs_max, std::memory_order_relaxed);
  }
  const int64_t tiles = ((a.m + 2 * kBM - 1) / (2 * kBM)) * ((a.n + BN - 1) / BN);
  const int pairs = int(tiles < pairs_max ? tiles : pairs_max);
  lc.gridDim = dim3(2 * unsigned(pairs));
  e = cudaLaunchKernelEx(&lc, kern, ta, tb, tc, int(a.m), int(a.n), int(a.k), cfg.group_m, ks::wait_ctx());
  if (e != cudaSuccess) return ks::map_cuda(e);
  return ks::map_cuda(cudaGetLastError());
}

template <int BN, int ACC>
int launch_tc2_stages(const ks_matmul_config &cfg, const ks_matmul_args &a, cudaStream_t st) {
  switch (cfg.stages) {
    case 2: return launch_tc2<BN, 2, ACC>(cfg, a, st);
    case 3: return launch_tc2<BN, 3, ACC>(cfg, a, st);
    case 4: return launch_tc2<BN, 4, ACC>(cfg, a, st);
    case 5: return launch_tc2<BN, 5, ACC>(cfg, a, st);
    case 6: return launch_tc2<BN, 6, ACC>(cfg, a, st);
    default: return KS_ERR_INVALID_CONFIG;
  }
}

// Stage counts instantiated per tile width (the ring must fit 227 KB).
template <int BN>
constexpr int max_stages() { return BN == 256 ? 4 : 6; }

template <int BN, int ACC>
int launch_tc_stages(const ks_matmul_config &cfg, const ks_matmul_args &a, cudaStream_t st) {
  switch (cfg.stages) {
    case 2: return launch_tc<BN, 2, ACC>(cfg, a, st);
    case 3: return launch_tc<BN, 3, ACC>(cfg, a, st);
    case 4: return launch_tc<BN, 4, ACC>(cfg, a, st);
    case 5: if constexpr (max_stages<BN>() >= 5) return launch_tc<BN, 5, ACC>(cfg, a, st);
      return KS_ERR_INVALID_CONFIG;
    case 6: if constexpr (max_stages<BN>() >= 6) return launch_tc<BN, 6, ACC>(cfg, a, st);
      return KS_ERR_INVALID_CONFIG;
    default: return KS_ERR_INVALID_CONFIG;
  }
}

// One CTA with 256-row tiles (two M=128 MMAs per B tile): the A ring holds
// two 128-row boxes per stage.  tile_n 256: stages 2-3, one accumulator
// (2 x 256 TMEM columns); tile_n 128: stages 2-4, one or two accumulators.
template <int BN, int ACC>
int launch_tc_wide_stages(const ks_matmul_config &cfg, const ks_matmul_args &a, cudaStream_t st) {
  switch (cfg.stages) {
    case 2: return launch_tc<BN, 2, ACC, 2>(cfg, a, st);
    case 3: return launch_tc<BN, 3, ACC, 2>(cfg, a, st);
    case 4: if constexpr (BN == 128) return launch_tc<BN, 4, ACC, 2>(cfg, a, st);
      return KS_ERR_INVALID_CONFIG;
    default: return KS_ERR_INVALID_CONFIG;
  }
}

constexpr uint32_t kSmemLimit = 227 * 1024;

// Per-CTA bytes: A ring (two 128-row boxes per stage for one-CTA 256-row
// tiles) + B ring (half of tile_n per CTA for the pair kernel) + the C
// staging buffers of the TMA-store epilogue + barriers + alignment slack.
uint32_t smem_for(int bm, int bn, int stages, int cta_group) {
  const bool pair = bm == 256 && cta_group != 1;
  const uint32_t a_bytes = bm == 256 && !pair ? 2 * kABytes : kABytes;
  const uint32_t b_cols = pair ? uint32_t(bn / 2) : uint32_t(bn);
  return uint32_t(stages) * (a_bytes + uint32_t(kBK) * b_cols * 2) + kCStage + (2 * stages + 7) * 8 + 16 + 1024;
}

}  // namespace

extern "C" {

int ks_matmul_validate(const ks_matmul_config *cfg, int64_t m, int64_t n, int64_t k, char *reason, size_t len) {
  if (!cfg) return KS_ERR_INVALID_ARGS;
  if (cfg->tile_m != 128 && cfg->tile_m != 256) {
    ks::set_reason(reason, len,
                   "matmul: tile_m must be 128 (one CTA, UMMA M=128) or 256 (a CTA pair, cta_group::2 M=256, or one "
                   "CTA with two M=128 MMAs)");
    return KS_ERR_INVALID_CONFIG;
  }
  if (cfg->cta_group < 0 || cfg->cta_group > 2 || (cfg->tile_m == 128 && cfg->cta_group == 2)) {
    ks::set_reason(reason, len, "matmul: cta_group must be 0 (default), 1, or 2 with tile_m 256");
    return KS_ERR_INVALID_CONFIG;
  }
  const bool wide = cfg->tile_m == 256 && cfg->cta_group == 1;  // one CTA, 256-row tiles
  if (cfg->tile_n != 64 && cfg->tile_n != 128 && cfg->tile_n != 256) {
    ks::set_reason(reason, len, "matmul: tile_n must be 64, 128 or 256 (sm_100a space)");
    return KS_ERR_INVALID_CONFIG;
  }
  if (cfg->tile_m == 256 && cfg->tile_n == 64) {
    ks::set_reason(reason, len,
                   "matmul: tile_m 256 needs tile_n 128 or 256 (a pair's CTA loads tile_n/2 >= 64 columns)");
    return KS_ERR_INVALID_CONFIG;
  }
  if (cfg->tile_k != 64) {
    ks::set_reason(reason, len, "matmul: tile_k must be 64 (one 128-byte swizzle row of bf16)");
    return KS_ERR_INVALID_CONFIG;
  }
  const int max_st = wide ? (cfg->tile_n == 256 ? 3 : 4) : (cfg->tile_n == 256 && cfg->tile_m == 128) ? 4 : 6;
  if (cfg->stages < 2 || cfg->stages > max_st) {
    ks::set_reason(reason, len, "matmul: stages must be 2..%d for tile %dx%d", max_st, cfg->tile_m, cfg->tile_n);
    return KS_ERR_INVALID_CONFIG;
  }
  if (cfg->acc_stages != 1 && cfg->acc_stages != 2) {
    ks::set_reason(reason, len, "matmul: acc_stages must be 1 or 2 (TMEM accumulator buffers)");
    return KS_ERR_INVALID_CONFIG;
  }
  if (wide && cfg->acc_stages * cfg->tile_n * 2 > 512) {
    ks::set_reason(reason, len, "matmul: a one-CTA 256x%d tile with %d accumulators needs %d > 512 TMEM columns",
                   cfg->tile_n, cfg->acc_stages, cfg->acc_stages * cfg->tile_n * 2);
    return KS_ERR_INVALID_CONFIG;
  }
  if (cfg->group_m < -32 || cfg->group_m == 0 || cfg->group_m > 64) {
    ks::set_reason(reason, len,
                   "matmul: group_m must be 1..64 (raster groups of M-tiles) or -32..-1 (bands of N-tiles, B kept "
                   "in L2)");
    return KS_ERR_INVALID_CONFIG;
  }
  const uint32_t smem = smem_for(cfg->tile_m, cfg->tile_n, cfg->stages, cfg->cta_group);
  if (smem > kSmemLimit) {
    ks::set_reason(reason, len, "matmul: %u bytes of shared memory for %d stages of %dx%dx64 > %u", smem,
                   cfg->stages, cfg->tile_m, cfg->tile_n, kSmemLimit);
    return KS_ERR_INVALID_CONFIG;
  }
  if (m < 0 || n < 0 || k < 0) {
    ks::set_reason(reason, len, "matmul: negative shape");
    return KS_ERR_INVALID_ARGS;
  }
  ks::set_reason(reason, len, "");
  return KS_OK;
}

int ks_matmul_launch(const ks_matmul_config *cfg, const ks_matmul_args *a, void *stream) {
  if (!cfg || !a) return KS_ERR_INVALID_ARGS;
  int s = ks_matmul_validate(cfg, a->m, a->n, a->k, nullptr, 0);
  if (s != KS_OK) return s;
  if (a->m == 0 || a->n == 0) return KS_OK;
  if (!a->out) return KS_ERR_INVALID_ARGS;
  if ((s = ks::check_arch_sm100()) != KS_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->k == 0)  // empty inner dimension: C = 0 (A and B may be null)
    return ks::map_cuda(cudaMemsetAsync(a->out, 0, size_t(a->m) * size_t(a->n) * 2, st));
  if (!a->a || !a->b) return KS_ERR_INVALID_ARGS;
  if (!tc_shape_ok(*a)) {
    if (a->m >= (1LL << 31) || a->n >= (1LL << 31) || a->k >= (1LL << 31)) return KS_ERR_INVALID_ARGS;
    dim3 grid(unsigned((a->n + 63) / 64), unsigned((a->m + 63) / 64));
    matmul_simt_kernel<<<grid, 256, 0, st>>>(static_cast<const uint16_t *>(a->a), static_cast<const uint16_t *>(a->b),
                                             static_cast<uint16_t *>(a->out), int(a->m), int(a->n), int(a->k));
    return ks::map_cuda(cudaGetLastError());
  }
  const bool two = cfg->acc_stages == 2;
  if (cfg->tile_m == 256 && cfg->cta_group == 1) {  // one CTA, two M=128 MMAs per B tile
    if (cfg->tile_n == 128) return two ? launch_tc_wide_stages<128, 2>(*cfg, *a, st) : launch_tc_wide_stages<128, 1>(*cfg, *a, st);
    return launch_tc_wide_stages<256, 1>(*cfg, *a, st);
  }
  if (cfg->tile_m == 256) {
    if (cfg->tile_n == 128) return two ? launch_tc2_stages<128, 2>(*cfg, *a, st) : launch_tc2_stages<128, 1>(*cfg, *a, st);
    return two ? launch_tc2_stages<256, 2>(*cfg, *a, st) : launch_tc2_stages<256, 1>(*cfg, *a, st);
  }
  switch (cfg->tile_n) {
    case 64: return two ? launch_tc_stages<64, 2>(*cfg, *a, st) : launch_tc_stages<64, 1>(*cfg, *a, st);
    case 128: return two ? launch_tc_stages<128, 2>(*cfg, *a, st) : launch_tc_stages<128, 1>(*cfg, *a, st);
    default: return two ? launch_tc_stages<256, 2>(*cfg, *a, st) : launch_tc_stages<256, 1>(*cfg, *a, st);
  }
}

}  // extern "C"
