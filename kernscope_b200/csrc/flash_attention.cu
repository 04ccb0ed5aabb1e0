// flash_attention.cu -- attention forward (causal or not) on the sm_100a
// tensor cores.
//
// The reference family (flash_attention_gen.cpp:255-404) is a scalar
// FlashAttention-lite: per Br-row query tile it walks Bc-row K/V tiles with
// the online softmax (m, l, O rescale), S in shared memory, scalar dot
// products.  Same algorithm here (Dao et al. 2022, online softmax), mapped to
// Blackwell:
//
//   * config tile_m 256 (fa_fwd_kernel): one CTA = one (batch*head,
//     256-query block) = two 128-row Q tiles; tile_m 128 (fa_fwd1_kernel,
//     further below): one Q tile with S double-buffered.  K/V walked in
//     128-row tiles through a 2-stage TMA ring;
//   * warp 8 (one lane): TMA producer (Q once, K_j and V_j per tile,
//     128-byte swizzle, 3-D maps [BH][N][d] so out-of-range rows read zeros);
//   * warp 9 (one lane): tcgen05.mma issuer.  TMEM columns: S0 [0,128),
//     S1 [128,256), O0 [256,384), O1 [384,512) (fp32, lane = query row).
//     Issue order per K/V tile j: PV0(j-1), S0(j), PV1(j-1), S1(j) -- each
//     S MMA reuses the TMEM of the P its own tile just consumed (tcgen05
//     MMAs of one thread execute in issue order), and each softmax warpgroup
//     works while the tensor core runs the other tile's MMAs;
//   * warps 0-3 / 4-7: softmax warpgroups for Q tile 0 / 1.  Thread t owns
//     query row t: tcgen05.ld of its 128 scores, causal / length mask only
//     on tiles that need it (warp-uniform test), row max with 3-input max in
//     independent chains, P = exp2(s*log2(e)/sqrt(d) - m) with the scale
//     folded into a packed f32x2 FMA, fp32 row sum in packed f32x2 partials,
//     P rounded to bf16 and written back into TMEM (columns [0,64) of its S
//     region, two bf16 per column) as the A operand of O += P V.  The pipeline
//     period is (softmax time + one P V and one Q K^T MMA), so the softmax's
//     issue count per element is what bounds the tensor-core utilisation.  O
//     is rescaled only when the running max grows by more than 2^8 (values
//     exp2(s - m) stay <= 256, exact in fp32/bf16 range); the final O / l is
//     rounded to bf16 once and stored;
//   * causal: tile 0 stops one K/V tile before tile 1 (its last tile is fully
//     masked) and its epilogue starts while tile 1's last MMAs run;
//   * persistent: one CTA per SM walks (query block, head) work items, the
//     heaviest query blocks of a head first; the next item's Q load and
//     first QK^T MMAs overlap the current item's epilogue.
//
// All waits are bounded (KsWait); teardown waits for outstanding TMA loads
// and MMAs before TMEM is freed.
#include <cmath>

#include "ks_common.cuh"

namespace {

constexpr int kTile = 128;               // query rows per tile, K/V rows per tile
constexpr int kD = 128;                  // head dim
constexpr int kThreads = 320;            // 8 softmax warps + producer + MMA
// The two-tile kernel runs three warpgroups: softmax (warps 0-3, 4-7) and a
// third whose warps 8 and 9 are the producer and the MMA issuer.  Launched
// at 168 registers per thread (65536 / 384, rounded to the allocation
// granule), the third warpgroup gives registers back and the softmax
// warpgroups take them: 128 x 88 + 256 x 208 = 64512 <= 384 x 168 = 64512,
// so the increase never waits on registers the block does not hold (88 keeps
// the persistent producer/MMA state, 208 the softmax row, free of spills).
constexpr int kThreads2 = 384;
constexpr int kRegsLow = 88, kRegsHigh = 208;
static_assert(128 * kRegsLow + 256 * kRegsHigh <= kThreads2 * 168, "register split exceeds the launch");
constexpr uint32_t kBox = 128 * 64 * 2;  // [128 rows x 64 cols] bf16 box = 16 KB
constexpr uint32_t kTileBytes = 2 * kBox;  // [128 x 128] tile = 32 KB
constexpr int kStages = 2;


// Epilogue staging: per softmax warp two [32 rows x 32 columns] bf16 blocks
// (64-byte rows, 64-byte swizzle), 2 KB each; 8 warps = 32 KB.
constexpr uint32_t kOBuf = 32 * 64;
constexpr uint32_t kOStage = 8 * 2 * kOBuf;

// Bytes of one [128 rows x D] bf16 tile: D / 64 boxes of 64 columns.
template <int D>
constexpr uint32_t tile_bytes() {
  return uint32_t(D / 64) * kBox;
}

template <int D>
struct FaLayout {
  static constexpr uint32_t kTB = tile_bytes<D>();
  static constexpr uint32_t q_off = 0;                      // Q0, Q1
  static constexpr uint32_t k_off = q_off + 2 * kTB;        // K[stages]
  static constexpr uint32_t v_off = k_off + kStages * kTB;  // V[stages]
  static constexpr uint32_t o_off = v_off + kStages * kTB;  // O staging for the TMA-store epilogue
  static constexpr uint32_t bar_off = o_off + kOStage;
  // q_full, k_full[2], v_full[2], kv_empty[2], s_full[2], p_full[2], o_full[2], drain, p_half[2],
  // o_empty[2], q_empty
  static constexpr uint32_t n_bars = 1 + 3 * kStages + 2 + 2 + 2 + 1 + 2 + 2 + 1;
  static constexpr uint32_t misc_off = bar_off + n_bars * 8;
  static constexpr uint32_t bytes = misc_off + 16;
  static constexpr uint32_t smem_request = bytes + 1024;
};

KS_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

KS_DEV float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}


// Packed pairs of fp32 (Blackwell f32x2 arithmetic: one instruction, two
// lanes' worth of FFMA/FADD), used to halve the issue cost of the softmax.
struct F2 {
  float x, y;
};
KS_DEV F2 fma2(F2 a, F2 b, F2 c) {
  F2 d;
  asm("{\n\t.reg .b64 A, B, C, D;\n\t"
      "mov.b64 A, {%2, %3};\n\tmov.b64 B, {%4, %5};\n\tmov.b64 C, {%6, %7};\n\t"
      "fma.rn.f32x2 D, A, B, C;\n\tmov.b64 {%0, %1}, D;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
KS_DEV F2 add2(F2 a, F2 b) {
  F2 d;
  asm("{\n\t.reg .b64 A, B, D;\n\t"
      "mov.b64 A, {%2, %3};\n\tmov.b64 B, {%4, %5};\n\t"
      "add.rn.f32x2 D, A, B;\n\tmov.b64 {%0, %1}, D;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

KS_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// S(tile g) = Q_g K_j^T: M=128, N=128 (keys), K=d=128 in 8 steps of 16.
// Q and K tiles are K-major: two 64-column boxes of 128 rows (16 KB apart),
// 128-byte rows, 8-row groups 1024 bytes apart.
template <int D = kD>
KS_DEV void issue_s(uint32_t d_tmem, uint32_t q_addr, uint32_t k_addr) {
  constexpr uint32_t idesc = ks_idesc_bf16_f32(128, 128, false, false);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t off = (kk >> 2) * kBox + (kk & 3) * 32;
    ks_umma_ss(d_tmem, ks_umma_desc_sw128(q_addr + off, 16, 1024), ks_umma_desc_sw128(k_addr + off, 16, 1024),
               idesc, kk > 0);
  }
}

// O(tile g) (+)= P_g V_j: M=128, N=d=128, K=128 keys in 8 steps of 16.
// P comes from TMEM (8 columns = 16 bf16 per step); V is MN-major: two
// 64-column boxes 16 KB apart (LBO), 8 key-rows 1024 bytes apart (SBO),
// 16 key-rows = 2048 bytes per step.
template <int D = kD>
KS_DEV void issue_pv(uint32_t o_tmem, uint32_t p_tmem, uint32_t v_addr, bool accumulate, int kk0 = 0,
                     int kk1 = kTile / 16) {
  constexpr uint32_t idesc = ks_idesc_bf16_f32(128, D, false, true);
#pragma unroll
  for (int kk = kk0; kk < kk1; ++kk)
    ks_umma_ts(o_tmem, p_tmem + kk * 8, ks_umma_desc_sw128(v_addr + kk * 2048, kBox, 1024), idesc,
               accumulate || kk > 0);
}

// Work item k of CTA c (persistent grid of G CTAs): items are (256-query
// block, batch*head) pairs ordered heaviest causal block first; round r hands
// CTA c item r*G + c on even rounds and r*G + (G-1-c) on odd ones, which
// evens out the per-CTA load of the decreasing causal item sizes.
struct FaItem {
  int q0, bh, n_kv, n_t0;
};
KS_DEV bool fa_item(int r, int c, int G, int num_items, int num_qb, int n_bh, int nq, int nk, int causal,
                    FaItem &it) {
  const int w = r * G + ((r & 1) ? G - 1 - c : c);
  if (w >= num_items) return false;
  // consecutive items share a head (its K/V stays in L2 while the CTAs
  // running them stream it), heaviest query block of the head first
  const int qb = num_qb - 1 - w % num_qb;
  it.bh = w / num_qb;
  it.q0 = qb * 2 * kTile;
  int n_kv = (nk + kTile - 1) / kTile;
  // tile g needs K/V tiles [0, n_t[g]); n_kv = n_t[1] >= n_t[0].  Under the
  // causal mask tile 0 stops one K/V tile earlier (its last one is masked).
  int n_t0 = n_kv;
  if (causal) {
    n_t0 = min(n_kv, (it.q0 + kTile - 1) / kTile + 1);
    const int q_last = min(it.q0 + 2 * kTile, nq) - 1;
    n_kv = min(n_kv, q_last / kTile + 1);
    n_t0 = min(n_t0, n_kv);
  }
  it.n_kv = n_kv;
  it.n_t0 = n_t0;
  return true;
}

// Persistent: one CTA per SM walks its work items; the next item's Q load
// and first QK^T MMAs run while the softmax warpgroups finish the current
// item's epilogue.  Phases of the per-step barriers continue across items.
template <int D>
__global__ void __launch_bounds__(kThreads2, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o, int nq, int nk,
                  int n_bh, float scale_log2, int causal, KsWait wait) {
  using L = FaLayout<D>;
  constexpr uint32_t kTB = L::kTB;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ks_smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::bar_off);
  uint64_t *q_full = bars;
  uint64_t *k_full = bars + 1;
  uint64_t *v_full = bars + 1 + kStages;
  uint64_t *kv_empty = bars + 1 + 2 * kStages;
  uint64_t *s_full = bars + 1 + 3 * kStages;
  uint64_t *p_full = s_full + 2;
  uint64_t *o_full = p_full + 2;
  uint64_t *drain = o_full + 2;
  uint64_t *p_half = drain + 1;
  uint64_t *o_empty = p_half + 2;
  uint64_t *q_empty = o_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::misc_off);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + L::misc_off + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_qb = (nq + 2 * kTile - 1) / (2 * kTile);
  const int num_items = num_qb * n_bh;
  const int cta = int(blockIdx.x), G = int(gridDim.x);

  if (threadIdx.x == 0) {
    ks_mbar_init(q_full, 1);
    ks_mbar_init(q_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      ks_mbar_init(k_full + s, 1);
      ks_mbar_init(v_full + s, 1);
      ks_mbar_init(kv_empty + s, 1);
    }
    for (int g = 0; g < 2; ++g) {
      ks_mbar_init(s_full + g, 1);
      ks_mbar_init(p_full + g, 4);
      ks_mbar_init(p_half + g, 4);
      ks_mbar_init(o_full + g, 1);
      ks_mbar_init(o_empty + g, 4);
    }
    ks_mbar_init(drain, 1);
    *abort = 0;
    ks_fence_mbar_init();
    ks_prefetch_tmap(&tm_q);
    ks_prefetch_tmap(&tm_k);
    ks_prefetch_tmap(&tm_v);
    ks_prefetch_tmap(&tm_o);
  }
  if (warp == 9) {
    ks_tmem_alloc(tmem_slot, 512);
    ks_tmem_relinquish();
  }
  ks_tc_fence_before();
  __syncthreads();
  ks_tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Registers move from the producer/MMA warpgroup to the softmax ones
  // (warpgroup-uniform branches; the roles stay inside them).
  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
    if (warp == 8) {
      if (lane == 0) {
        // ---------------------------------------------------------- producer
        uint8_t *qs = smem + L::q_off;
        uint32_t armed = 0, armed_par = 0;
        int gj = 0;       // K/V tiles loaded so far (ring position)
        int q_loads = 0;  // Q tile pairs loaded so far
        bool ok = true;
        FaItem it;
        for (int r = 0; ok && fa_item(r, cta, G, num_items, num_qb, n_bh, nq, nk, causal, it); ++r) {
          // the previous item's last QK^T MMA has read Q
          if (r > 0 && !ks_mbar_wait(q_empty, (r - 1) & 1, abort, wait)) break;
          ks_mbar_arrive_expect_tx(q_full, 2 * kTB);
          for (int g = 0; g < 2; ++g)
            for (int h = 0; h < D / 64; ++h)
              ks_tma_load_3d(qs + g * kTB + h * kBox, &tm_q, q_full, h * 64, it.q0 + g * kTile, it.bh);
          ++q_loads;
          for (int j = 0; j < it.n_kv; ++j, ++gj) {
            const int st = gj % kStages;
            const uint32_t ph = (gj / kStages) & 1;
            if (!ks_mbar_wait(kv_empty + st, ph ^ 1u, abort, wait)) {
              ok = false;
              break;
            }
            uint8_t *ks = smem + L::k_off + st * kTB;
            uint8_t *vs = smem + L::v_off + st * kTB;
            ks_mbar_arrive_expect_tx(k_full + st, kTB);
            for (int h = 0; h < D / 64; ++h)
              ks_tma_load_3d(ks + h * kBox, &tm_k, k_full + st, h * 64, j * kTile, it.bh);
            ks_mbar_arrive_expect_tx(v_full + st, kTB);
            for (int h = 0; h < D / 64; ++h)
              ks_tma_load_3d(vs + h * kBox, &tm_v, v_full + st, h * 64, j * kTile, it.bh);
            armed |= 1u << st;
            armed_par = (armed_par & ~(1u << st)) | (ph << st);
          }
        }
        // teardown: the loads issued above have landed (the last Q and the
        // last K/V of each ring stage)
        if (q_loads > 0) ks_mbar_wait(q_full, (q_loads - 1) & 1, nullptr, wait);
        for (int s = 0; s < kStages; ++s)
          if (armed & (1u << s)) {
            ks_mbar_wait(k_full + s, (armed_par >> s) & 1u, nullptr, wait);
            ks_mbar_wait(v_full + s, (armed_par >> s) & 1u, nullptr, wait);
          }
      }
    } else if (warp == 9) {
      if (lane == 0) {
        // ---------------------------------------------------------- MMA issuer
        const uint32_t q_addr = ks_smem_u32(smem + L::q_off);
        const uint32_t k_addr = ks_smem_u32(smem + L::k_off);
        const uint32_t v_addr = ks_smem_u32(smem + L::v_off);
        const uint32_t t_s[2] = {tmem + 0, tmem + 128};
        const uint32_t t_o[2] = {tmem + 256, tmem + 384};
        int gj = 0;           // K/V tiles consumed so far (ring position)
        int sg[2] = {0, 0};   // steps of each tile so far (s_full / p_half / p_full phases)
        bool ok = true;
        FaItem it;
        for (int r = 0; ok && fa_item(r, cta, G, num_items, num_qb, n_bh, nq, nk, causal, it); ++r) {
          const int n_t[2] = {it.n_t0, it.n_kv};
          if (!ks_mbar_wait(q_full, r & 1, abort, wait) ||
              !ks_mbar_wait(k_full + gj % kStages, (gj / kStages) & 1, abort, wait))
            break;
          ks_tc_fence_after();
          issue_s<D>(t_s[0], q_addr, k_addr + (gj % kStages) * kTB);
          ks_umma_commit(s_full + 0);
          issue_s<D>(t_s[1], q_addr + kTB, k_addr + (gj % kStages) * kTB);
          ks_umma_commit(s_full + 1);
          if (it.n_kv == 1) ks_umma_commit(q_empty);  // that was the item's last read of Q
          for (int j = 0; j < it.n_kv && ok; ++j, ++gj) {
            const int st = gj % kStages;
            const uint32_t ph = (gj / kStages) & 1;
            const int st1 = (gj + 1) % kStages;
            const uint32_t ph1 = ((gj + 1) / kStages) & 1;
            const bool more0 = j + 1 < n_t[0], more1 = j + 1 < it.n_kv;
            ok = false;
            if (!ks_mbar_wait(v_full + st, ph, abort, wait)) break;
            // the first P V of an item overwrites O: the previous item's
            // epilogue must have read it
            if (j == 0 && r > 0 &&
                (!ks_mbar_wait(o_empty + 0, (r - 1) & 1, abort, wait) ||
                 !ks_mbar_wait(o_empty + 1, (r - 1) & 1, abort, wait)))
              break;
            // tile 0: O0 += P0 V_j, then S0 = Q0 K_{j+1}^T into the freed TMEM
            if (j < n_t[0]) {
              // the first half of P (keys 0-63) is read while the softmax stores the second
              if (!ks_mbar_wait(p_half + 0, sg[0] & 1, abort, wait)) break;
              ks_tc_fence_after();
              issue_pv<D>(t_o[0], t_s[0], v_addr + st * kTB, j > 0, 0, 4);
              if (!ks_mbar_wait(p_full + 0, sg[0] & 1, abort, wait)) break;
              ks_tc_fence_after();
              issue_pv<D>(t_o[0], t_s[0], v_addr + st * kTB, true, 4, 8);
              ++sg[0];
              if (j + 1 == n_t[0]) ks_umma_commit(o_full + 0);
            }
            if (more1) {
              if (!ks_mbar_wait(k_full + st1, ph1, abort, wait)) break;
              ks_tc_fence_after();
            }
            if (more0) {
              issue_s<D>(t_s[0], q_addr, k_addr + st1 * kTB);
              ks_umma_commit(s_full + 0);
            }
            // tile 1
            if (!ks_mbar_wait(p_half + 1, sg[1] & 1, abort, wait)) break;
            ks_tc_fence_after();
            issue_pv<D>(t_o[1], t_s[1], v_addr + st * kTB, j > 0, 0, 4);
            if (!ks_mbar_wait(p_full + 1, sg[1] & 1, abort, wait)) break;
            ks_tc_fence_after();
            issue_pv<D>(t_o[1], t_s[1], v_addr + st * kTB, true, 4, 8);
            ++sg[1];
            ks_umma_commit(kv_empty + st);
            if (more1) {
              issue_s<D>(t_s[1], q_addr + kTB, k_addr + st1 * kTB);
              ks_umma_commit(s_full + 1);
              if (j + 2 == it.n_kv) ks_umma_commit(q_empty);  // the item's last read of Q
            } else {
              ks_umma_commit(o_full + 1);
            }
            ok = true;
          }
        }
        ks_umma_commit(drain);
        ks_mbar_wait(drain, 0, nullptr, wait);
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
    // ------------------------------------------------------------ softmax
    const int g = warp >> 2;         // Q tile of this warpgroup
    const int qd = warp & 3;         // TMEM lane quadrant
    const int row = qd * 32 + lane;  // row within the tile = TMEM lane
    const uint32_t lane_addr = tmem + (uint32_t(qd * 32) << 16);
    const uint32_t s_col = g * 128, o_col = 256 + g * 128;
    uint32_t nstore = 0;  // epilogue blocks stored (staging buffer = nstore & 1)
    int sg = 0;  // steps of this tile so far, over all items
    bool ok = true;
    FaItem it;
    for (int r = 0; ok && fa_item(r, cta, G, num_items, num_qb, n_bh, nq, nk, causal, it); ++r) {
      const int qrow = it.q0 + g * kTile + row;
      float m = -INFINITY, l = 0.f;
      const int n_mine = g == 0 ? it.n_t0 : it.n_kv;
      for (int j = 0; j < n_mine; ++j, ++sg) {
        if (!ks_mbar_wait(s_full + g, sg & 1, abort, wait)) {
          ok = false;
          break;
        }
        ks_tc_fence_after();
        uint32_t rr[128];
        ks_tmem_ld32_at<0>(lane_addr + s_col + 0, rr);
        ks_tmem_ld32_at<32>(lane_addr + s_col + 32, rr);
        ks_tmem_ld32_at<64>(lane_addr + s_col + 64, rr);
        ks_tmem_ld32_at<96>(lane_addr + s_col + 96, rr);
        ks_tmem_wait_ld();
        const int kv0 = j * kTile;
        // keys beyond this row's limit are masked: causal (key > query) and length
        int lim = nk - kv0;  // number of valid keys in this tile
        if (causal) lim = min(lim, qrow - kv0 + 1);
        // warp-uniform: most tiles are unmasked for all 32 rows of the warp
        const bool full_tile = __all_sync(0xffffffffu, lim >= kTile);
        if (!full_tile) {
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c >= lim) rr[c] = 0xff800000u;  // -inf
        }
        // row max of the raw scores (scale > 0 commutes with max), as four
        // independent chains of 3-input max so latency does not serialise
        float mm[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          mm[u] = max3(__uint_as_float(rr[u]), __uint_as_float(rr[u + 4]), __uint_as_float(rr[u + 8]));
#pragma unroll
        for (int c = 12; c < 124; c += 8)
#pragma unroll
          for (int u = 0; u < 4; ++u)
            mm[u] = max3(mm[u], __uint_as_float(rr[c + u]), __uint_as_float(rr[c + 4 + u]));
#pragma unroll
        for (int u = 0; u < 4; ++u) mm[u] = fmaxf(mm[u], __uint_as_float(rr[124 + u]));
        const float mx = fmaxf(fmaxf(mm[0], mm[1]), fmaxf(mm[2], mm[3]));
        const float m_new = fmaxf(m, mx * scale_log2);
        const bool grow = m_new > m + 8.f;  // also true on the first finite max
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
          // O has absorbed every earlier P V of this item (the S commit
          // follows it), rescale.
          const float alpha = grow ? ex2(m - m_new) : 1.f;
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            ks_tmem_ld32(lane_addr + o_col + c * 32, o);
            ks_tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(lane_addr + o_col + c * 32, o);
          }
          ks_tmem_wait_st();
        }
        if (grow) {
          l *= ex2(m - m_new);
          m = m_new;
        }
        const float neg_m = (m == -INFINITY) ? 0.f : -m;
        F2 rsum[4] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};  // independent partial sums
        const F2 sc2{scale_log2, scale_log2}, nm2{neg_m, neg_m};
        // P in two halves of 64 keys (32 packed columns each), stored over S
        // columns already in registers.  The first half is announced (p_half)
        // once the second is computed, so the tensor core starts O += P V on
        // keys 0-63 while the second half is stored.
        uint32_t p[2][32];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int e0 = 64 * half + 2 * c;
            // exponent pair x = s*scale_log2 - m as one packed FFMA
            const F2 x = fma2(F2{__uint_as_float(rr[e0]), __uint_as_float(rr[e0 + 1])}, sc2, nm2);
            const F2 e{ex2(x.x), ex2(x.y)};
            rsum[c & 3] = add2(rsum[c & 3], e);
            p[half][c] = ks_pack_bf16x2(e.x, e.y);
          }
          if (half == 0) ks_tmem_st32_at<0>(lane_addr + s_col + 0, p[0]);
        }
        ks_tmem_wait_st();
        ks_tc_fence_before();
        __syncwarp();
        if (lane == 0) ks_mbar_arrive(p_half + g);
        ks_tmem_st32_at<0>(lane_addr + s_col + 32, p[1]);
        const F2 rs2 = add2(add2(rsum[0], rsum[1]), add2(rsum[2], rsum[3]));
        l += rs2.x + rs2.y;
        ks_tmem_wait_st();
        ks_tc_fence_before();
        __syncwarp();
        if (lane == 0) ks_mbar_arrive(p_full + g);
      }
      // epilogue: O / l -> bf16, 32 columns at a time through this warp's two
      // swizzled staging blocks, stored with TMA (rows >= nq are clipped);
      // O is free again once its last columns are in registers
      if (!ok || !ks_mbar_wait(o_full + g, r & 1, abort, wait)) {
        ok = false;
        break;
      }
      ks_tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint8_t *ostg = smem + L::o_off + warp * 2 * kOBuf;  // this warp's two staging blocks
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        ks_tmem_ld32(lane_addr + o_col + c * 32, o);
        ks_tmem_wait_ld();
        if (c + 1 == D / 32) {
          ks_tc_fence_before();
          __syncwarp();
          if (lane == 0) ks_mbar_arrive(o_empty + g);
        }
        uint8_t *buf = ostg + (nstore & 1) * kOBuf;
        if (lane == 0) ks_bulk_wait_read<1>();  // the store two blocks back has read this buffer
        __syncwarp();
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          w.x = ks_pack_bf16x2(__uint_as_float(o[v * 8 + 0]) * inv, __uint_as_float(o[v * 8 + 1]) * inv);
          w.y = ks_pack_bf16x2(__uint_as_float(o[v * 8 + 2]) * inv, __uint_as_float(o[v * 8 + 3]) * inv);
          w.z = ks_pack_bf16x2(__uint_as_float(o[v * 8 + 4]) * inv, __uint_as_float(o[v * 8 + 5]) * inv);
          w.w = ks_pack_bf16x2(__uint_as_float(o[v * 8 + 6]) * inv, __uint_as_float(o[v * 8 + 7]) * inv);
          *reinterpret_cast<uint4 *>(buf + lane * 64 + ((v ^ ((lane >> 1) & 3)) * 16)) = w;
        }
        ks_fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          ks_tma_store_3d(&tm_o, buf, c * 32, it.q0 + g * kTile + qd * 32, it.bh);
          ks_bulk_commit_group();
        }
        ++nstore;
      }
    }
    if (lane == 0) ks_bulk_wait_all();  // O is in global memory before the CTA exits
  }

  ks_tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    ks_tc_fence_after();
    ks_tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Two Q tiles per CTA with S in 64-key slots (config tile_m 256, tile_n 64).
//
// In the kernel above each tile computes S for 128 keys into the TMEM that
// P of the previous 128 keys occupies, so a tile's chain per K/V tile is
// softmax -> P V -> next Q K^T -> softmax, and the tensor core waits out the
// hand-over.  Here each tile's 128 S columns are two 64-column slots and
// every 64-key half-block is one online-softmax step (its own row max and
// rescale check, P written over its slot, O += P V with K = 64).  The next
// Q K^T of a slot is issued as soon as P V has read that slot, so it runs
// while the softmax works on the other slot: the tile's chain per half-block
// is one softmax step plus the hand-over, and the MMAs fill the gaps.
//
// TMEM: tile g's slots at columns [128 g, 128 g + 64) and [128 g + 64,
// 128 g + 128), O_g at [256 + 128 g, 256 + 128 g + 128).  Half-step h of a
// tile covers keys [64 h, 64 h + 64) of K/V tile h / 2 and uses slot h % 2.
// K and V stages are released separately (K after the last Q K^T reading
// it, two half-steps before V), so the loads run further ahead.  A rescale
// of O at step h waits for the tile's P V of step h - 1 (barrier pv_done).
// ---------------------------------------------------------------------------
template <int D>
struct FaRingLayout {
  static constexpr uint32_t kTB = tile_bytes<D>();
  static constexpr uint32_t q_off = 0;                      // Q0, Q1
  static constexpr uint32_t k_off = q_off + 2 * kTB;        // K[stages]
  static constexpr uint32_t v_off = k_off + kStages * kTB;  // V[stages]
  static constexpr uint32_t bar_off = v_off + kStages * kTB;
  // q_full, q_empty, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2][2], p_full[2][2],
  // pv_done[2], o_full[2], o_empty[2], drain
  static constexpr uint32_t n_bars = 2 + 4 * kStages + 4 + 4 + 2 + 2 + 2 + 1;
  static constexpr uint32_t misc_off = bar_off + n_bars * 8;
  static constexpr uint32_t bytes = misc_off + 16;
  static constexpr uint32_t smem_request = bytes + 1024;
};

// S(slot) = Q_g K_half^T: M=128, N=64 keys, K=d in steps of 16.  The K
// half-tile starts 64 rows (8192 bytes, eight 1024-byte swizzle groups) into
// each 64-column box.
template <int D>
KS_DEV void issue_s_half(uint32_t d_tmem, uint32_t q_addr, uint32_t k_half_addr) {
  constexpr uint32_t idesc = ks_idesc_bf16_f32(128, 64, false, false);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t off = (kk >> 2) * kBox + (kk & 3) * 32;
    ks_umma_ss(d_tmem, ks_umma_desc_sw128(q_addr + off, 16, 1024),
               ks_umma_desc_sw128(k_half_addr + off, 16, 1024), idesc, kk > 0);
  }
}

// O_g (+)= P(slot) V_half: M=128, N=d, K=64 keys in 4 steps of 16; P is the
// slot's first 32 columns (two bf16 per column), V_half starts 64 key-rows
// (8192 bytes) into the MN-major tile.
template <int D>
KS_DEV void issue_pv_half(uint32_t o_tmem, uint32_t p_tmem, uint32_t v_half_addr, bool accumulate) {
  constexpr uint32_t idesc = ks_idesc_bf16_f32(128, D, false, true);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    ks_umma_ts(o_tmem, p_tmem + kk * 8, ks_umma_desc_sw128(v_half_addr + kk * 2048, kBox, 1024), idesc,
               accumulate || kk > 0);
}

template <int D>
__global__ void __launch_bounds__(kThreads2, 1)
    fa_ring_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, uint16_t *__restrict__ out, int nq, int nk,
                   int n_bh, float scale_log2, int causal, KsWait wait) {
  using L = FaRingLayout<D>;
  constexpr uint32_t kTB = L::kTB;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ks_smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::bar_off);
  uint64_t *q_full = bars;
  uint64_t *q_empty = bars + 1;
  uint64_t *k_full = bars + 2;
  uint64_t *k_empty = k_full + kStages;
  uint64_t *v_full = k_empty + kStages;
  uint64_t *v_empty = v_full + kStages;
  uint64_t *s_full = v_empty + kStages;  // [tile][slot]
  uint64_t *p_full = s_full + 4;         // [tile][slot]
  uint64_t *pv_done = p_full + 4;
  uint64_t *o_full = pv_done + 2;
  uint64_t *o_empty = o_full + 2;
  uint64_t *drain = o_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::misc_off);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + L::misc_off + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_qb = (nq + 2 * kTile - 1) / (2 * kTile);
  const int num_items = num_qb * n_bh;
  const int cta = int(blockIdx.x), G = int(gridDim.x);

  if (threadIdx.x == 0) {
    ks_mbar_init(q_full, 1);
    ks_mbar_init(q_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      ks_mbar_init(k_full + s, 1);
      ks_mbar_init(k_empty + s, 1);
      ks_mbar_init(v_full + s, 1);
      ks_mbar_init(v_empty + s, 1);
    }
    for (int i = 0; i < 4; ++i) {
      ks_mbar_init(s_full + i, 1);
      ks_mbar_init(p_full + i, 4);
    }
    for (int g = 0; g < 2; ++g) {
      ks_mbar_init(pv_done + g, 1);
      ks_mbar_init(o_full + g, 1);
      ks_mbar_init(o_empty + g, 4);
    }
    ks_mbar_init(drain, 1);
    *abort = 0;
    ks_fence_mbar_init();
    ks_prefetch_tmap(&tm_q);
    ks_prefetch_tmap(&tm_k);
    ks_prefetch_tmap(&tm_v);
  }
  if (warp == 9) {
    ks_tmem_alloc(tmem_slot, 512);
    ks_tmem_relinquish();
  }
  ks_tc_fence_before();
  __syncthreads();
  ks_tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
    if (warp == 8) {
      if (lane == 0) {
        // ---------------------------------------------------------- producer
        uint8_t *qs = smem + L::q_off;
        uint32_t k_armed = 0, k_par = 0, v_armed = 0, v_par = 0;
        int gj = 0, q_loads = 0;
        bool ok = true;
        FaItem it;
        for (int r = 0; ok && fa_item(r, cta, G, num_items, num_qb, n_bh, nq, nk, causal, it); ++r) {
          if (r > 0 && !ks_mbar_wait(q_empty, (r - 1) & 1, abort, wait)) break;
          ks_mbar_arrive_expect_tx(q_full, 2 * kTB);
          for (int g = 0; g < 2; ++g)
            for (int h = 0; h < D / 64; ++h)
              ks_tma_load_3d(qs + g * kTB + h * kBox, &tm_q, q_full, h * 64, it.q0 + g * kTile, it.bh);
          ++q_loads;
          for (int j = 0; j < it.n_kv; ++j, ++gj) {
            const int st = gj % kStages;
            const uint32_t ph = (gj / kStages) & 1;
            if (!ks_mbar_wait(k_empty + st, ph ^ 1u, abort, wait)) {
              ok = false;
              break;
            }
            ks_mbar_arrive_expect_tx(k_full + st, kTB);
            for (int h = 0; h < D / 64; ++h)
              ks_tma_load_3d(smem + L::k_off + st * kTB + h * kBox, &tm_k, k_full + st, h * 64, j * kTile, it.bh);
            k_armed |= 1u << st;
            k_par = (k_par & ~(1u << st)) | (ph << st);
            if (!ks_mbar_wait(v_empty + st, ph ^ 1u, abort, wait)) {
              ok = false;
              break;
            }
            ks_mbar_arrive_expect_tx(v_full + st, kTB);
            for (int h = 0; h < D / 64; ++h)
              ks_tma_load_3d(smem + L::v_off + st * kTB + h * kBox, &tm_v, v_full + st, h * 64, j * kTile, it.bh);
            v_armed |= 1u << st;
            v_par = (v_par & ~(1u << st)) | (ph << st);
          }
        }
        // teardown: the loads issued above have landed
        if (q_loads > 0) ks_mbar_wait(q_full, (q_loads - 1) & 1, nullptr, wait);
        for (int s = 0; s < kStages; ++s) {
          if (k_armed & (1u << s)) ks_mbar_wait(k_full + s, (k_par >> s) & 1u, nullptr, wait);
          if (v_armed & (1u << s)) ks_mbar_wait(v_full + s, (v_par >> s) & 1u, nullptr, wait);
        }
      }
    } else if (warp == 9) {
      if (lane == 0) {
        // ---------------------------------------------------------- MMA issuer
        const uint32_t q_addr = ks_smem_u32(smem + L::q_off);
        const uint32_t k_addr = ks_smem_u32(smem + L::k_off);
        const uint32_t v_addr = ks_smem_u32(smem + L::v_off);
        int gj = 0;                     // K/V tiles consumed so far (ring position)
        uint32_t par0 = 0, par1 = 0;    // p_full phase parities of tile 0 / 1, bit = slot
        bool ok = true;
        FaItem it;
        for (int r = 0; ok && fa_item(r, cta, G, num_items, num_qb, n_bh, nq, nk, causal, it); ++r) {
          const int H0 = 2 * it.n_t0, H1 = 2 * it.n_kv;  // half-steps per tile; H1 >= H0
          ok = false;
          if (!ks_mbar_wait(q_full, r & 1, abort, wait) ||
              !ks_mbar_wait(k_full + gj % kStages, (gj / kStages) & 1, abort, wait))
            break;
          ks_tc_fence_after();
          // prologue: both slots of both tiles from K/V tile 0
#pragma unroll
          for (int g = 0; g < 2; ++g)
#pragma unroll
            for (int s = 0; s < 2; ++s) {  // H0, H1 >= 2
              issue_s_half<D>(tmem + g * 128 + s * 64, q_addr + g * kTB, k_addr + (gj % kStages) * kTB + s * 8192);
              ks_umma_commit(s_full + 2 * g + s);
            }
          ks_umma_commit(k_empty + gj % kStages);  // K tile 0 is fully read
          if (H1 <= 2) ks_umma_commit(q_empty);     // that was the item's last read of Q
          ok = true;
          for (int h = 0; h < H1 && ok; ++h) {
            const int half = h & 1;
            const int jj = gj + (h >> 1);  // ring position of this step's K/V tile
            const int st = jj % kStages;
            const int jn = jj + 1, stn = jn % kStages;
            ok = false;
            if (half == 0 && !ks_mbar_wait(v_full + st, (jj / kStages) & 1, abort, wait)) break;
            // this step's Q K^T (half-step h + 2) reads K tile jn, loaded three half-steps ago
            if (h + 2 < H1 && !ks_mbar_wait(k_full + stn, (jn / kStages) & 1, abort, wait)) break;
            ks_tc_fence_after();
            // one half-step of tile g: O_g += P V, then the slot's next Q K^T
            // (half-step h + 2 reads K/V tile jn); false on a failed wait
            auto step = [&](int g, int hg, uint32_t &uses) -> bool {
              if (h >= hg) return true;
              // the item's first P V overwrites O: the previous epilogue must have read it
              if (h == 0 && r > 0 && !ks_mbar_wait(o_empty + g, (r - 1) & 1, abort, wait)) return false;
              if (!ks_mbar_wait(p_full + 2 * g + half, (uses >> half) & 1u, abort, wait)) return false;
              uses ^= 1u << half;
              ks_tc_fence_after();
              issue_pv_half<D>(tmem + 256 + g * 128, tmem + g * 128 + half * 64, v_addr + st * kTB + half * 8192,
                               h > 0);
              ks_umma_commit(pv_done + g);
              if (h + 1 == hg) ks_umma_commit(o_full + g);
              if (h + 2 < hg) {
                issue_s_half<D>(tmem + g * 128 + half * 64, q_addr + g * kTB, k_addr + stn * kTB + half * 8192);
                ks_umma_commit(s_full + 2 * g + half);
              }
              return true;
            };
            if (!step(0, H0, par0) || !step(1, H1, par1)) break;
            if (half == 1) {
              ks_umma_commit(v_empty + st);                                 // V tile jj fully read
              if ((h >> 1) + 1 < it.n_kv) ks_umma_commit(k_empty + stn);  // so is K tile jn
            }
            if (h + 3 == H1) ks_umma_commit(q_empty);  // the item's last Q K^T was just issued
            ok = true;
          }
          gj += it.n_kv;
        }
        ks_umma_commit(drain);
        ks_mbar_wait(drain, 0, nullptr, wait);
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
    // ------------------------------------------------------------ softmax
    const int g = warp >> 2;         // Q tile of this warpgroup
    const int qd = warp & 3;         // TMEM lane quadrant
    const int row = qd * 32 + lane;  // row within the tile = TMEM lane
    const uint32_t lane_addr = tmem + (uint32_t(qd * 32) << 16);
    const uint32_t s_col = g * 128, o_col = 256 + g * 128;
    uint32_t spar = 0;  // s_full phase parity per slot (bit = slot), over all items
    int pv_base = 0;    // P V steps of this tile before the current item
    bool ok = true;
    FaItem it;
    for (int r = 0; ok && fa_item(r, cta, G, num_items, num_qb, n_bh, nq, nk, causal, it); ++r) {
      const int qrow = it.q0 + g * kTile + row;
      float m = -INFINITY, l = 0.f;
      const int Hg = 2 * (g == 0 ? it.n_t0 : it.n_kv);
      for (int h = 0; h < Hg; ++h) {
        const int slot = h & 1;
        if (!ks_mbar_wait(s_full + 2 * g + slot, (spar >> slot) & 1u, abort, wait)) {
          ok = false;
          break;
        }
        spar ^= 1u << slot;
        ks_tc_fence_after();
        uint32_t rr[64];
        ks_tmem_ld32_at<0>(lane_addr + s_col + slot * 64, rr);
        ks_tmem_ld32_at<32>(lane_addr + s_col + slot * 64 + 32, rr);
        ks_tmem_wait_ld();
        const int kv0 = h * 64;
        int lim = nk - kv0;  // valid keys of this half-block for this row
        if (causal) lim = min(lim, qrow - kv0 + 1);
        const bool full_block = __all_sync(0xffffffffu, lim >= 64);
        if (!full_block) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c >= lim) rr[c] = 0xff800000u;  // -inf
        }
        float mm[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          mm[u] = max3(__uint_as_float(rr[u]), __uint_as_float(rr[u + 4]), __uint_as_float(rr[u + 8]));
#pragma unroll
        for (int c = 12; c < 60; c += 8)
#pragma unroll
          for (int u = 0; u < 4; ++u)
            mm[u] = max3(mm[u], __uint_as_float(rr[c + u]), __uint_as_float(rr[c + 4 + u]));
#pragma unroll
        for (int u = 0; u < 4; ++u) mm[u] = fmaxf(mm[u], __uint_as_float(rr[60 + u]));
        const float mx = fmaxf(fmaxf(mm[0], mm[1]), fmaxf(mm[2], mm[3]));
        const float m_new = fmaxf(m, mx * scale_log2);
        const bool grow = m_new > m + 8.f;  // also true on the first finite max
        if (h > 0 && __any_sync(0xffffffffu, grow)) {
          // O must hold every earlier P V of this item before it is rescaled
          if (!ks_mbar_wait(pv_done + g, (pv_base + h - 1) & 1, abort, wait)) {
            ok = false;
            break;
          }
          ks_tc_fence_after();
          const float alpha = grow ? ex2(m - m_new) : 1.f;
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            ks_tmem_ld32(lane_addr + o_col + c * 32, o);
            ks_tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(lane_addr + o_col + c * 32, o);
          }
          ks_tmem_wait_st();
        }
        if (grow) {
          l *= ex2(m - m_new);
          m = m_new;
        }
        const float neg_m = (m == -INFINITY) ? 0.f : -m;
        F2 rsum[4] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
        const F2 sc2{scale_log2, scale_log2}, nm2{neg_m, neg_m};
        uint32_t p[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const F2 x = fma2(F2{__uint_as_float(rr[2 * c]), __uint_as_float(rr[2 * c + 1])}, sc2, nm2);
          const F2 e{ex2(x.x), ex2(x.y)};
          rsum[c & 3] = add2(rsum[c & 3], e);
          p[c] = ks_pack_bf16x2(e.x, e.y);
        }
        ks_tmem_st32_at<0>(lane_addr + s_col + slot * 64, p);
        const F2 rs2 = add2(add2(rsum[0], rsum[1]), add2(rsum[2], rsum[3]));
        l += rs2.x + rs2.y;
        ks_tmem_wait_st();
        ks_tc_fence_before();
        __syncwarp();
        if (lane == 0) ks_mbar_arrive(p_full + 2 * g + slot);
      }
      pv_base += Hg;
      // epilogue: O / l -> bf16 -> out[bh, qrow, :], then O is free again
      if (!ok || !ks_mbar_wait(o_full + g, r & 1, abort, wait)) {
        ok = false;
        break;
      }
      ks_tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint16_t *dst = out + (int64_t(it.bh) * nq + qrow) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        ks_tmem_ld32(lane_addr + o_col + c * 32, o);
        ks_tmem_wait_ld();
        if (qrow < nq) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = ks_pack_bf16x2(__uint_as_float(o[v * 8 + 0]) * inv, __uint_as_float(o[v * 8 + 1]) * inv);
            w.y = ks_pack_bf16x2(__uint_as_float(o[v * 8 + 2]) * inv, __uint_as_float(o[v * 8 + 3]) * inv);
            w.z = ks_pack_bf16x2(__uint_as_float(o[v * 8 + 4]) * inv, __uint_as_float(o[v * 8 + 5]) * inv);
            w.w = ks_pack_bf16x2(__uint_as_float(o[v * 8 + 6]) * inv, __uint_as_float(o[v * 8 + 7]) * inv);
            *reinterpret_cast<uint4 *>(dst + c * 32 + v * 8) = w;
          }
        }
      }
      ks_tc_fence_before();
      __syncwarp();
      if (lane == 0) ks_mbar_arrive(o_empty + g);
    }
  }

  ks_tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    ks_tc_fence_after();
    ks_tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// One 128-row Q tile per CTA with S double-buffered in TMEM.
//
// TMEM: S[0] columns [0,128), S[1] [128,256), O [256,384).  Because S(j+2)
// reuses the region of S(j) rather than the one being read, the tensor core
// computes S(j+1) while the softmax works on S(j): the MMA issue order is
// S(0), S(1), then per K/V tile j: O += P(j) V(j), S(j+2).  The two softmax
// warpgroups split each S tile by columns (keys [0,64) and [64,128)): both
// hold all 128 rows, exchange their partial row maxima through shared
// memory once per tile, keep partial row sums, and write their half of P
// (packed bf16) over the S columns they have read: keys [0,64) into columns
// [0,32), keys [64,128) into [64,96).  Each warpgroup rescales its half of
// O (64 of the 128 head-dim columns) when the running max grows by more than
// 2^8, after the previous P V has completed.  The pipeline period is the
// longer of the softmax time and one tile's two MMAs (S and P V).
// ---------------------------------------------------------------------------
struct Fa1Layout {
  static constexpr uint32_t q_off = 0;
  static constexpr uint32_t k_off = q_off + kTileBytes;
  static constexpr uint32_t v_off = k_off + kStages * kTileBytes;
  static constexpr uint32_t red_off = v_off + kStages * kTileBytes;  // float [2 steps][2 WGs][128 rows]
  static constexpr uint32_t lsum_off = red_off + 2 * 2 * 128 * 4;    // float [2 WGs][128 rows]
  static constexpr uint32_t bar_off = lsum_off + 2 * 128 * 4;
  // q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], p_full, pv_done, o_full, red, drain
  static constexpr uint32_t n_bars = 1 + 4 * kStages + 2 + 5;
  static constexpr uint32_t misc_off = bar_off + n_bars * 8;
  static constexpr uint32_t bytes = misc_off + 16;
  static constexpr uint32_t smem_request = bytes + 1024;
};

// O += P V for the split P layout above.
KS_DEV void issue_pv_split(uint32_t o_tmem, uint32_t s_tmem, uint32_t v_addr, bool accumulate) {
  constexpr uint32_t idesc = ks_idesc_bf16_f32(128, 128, false, true);
#pragma unroll
  for (int kk = 0; kk < kTile / 16; ++kk)
    ks_umma_ts(o_tmem, s_tmem + (kk < 4 ? kk * 8 : 64 + (kk - 4) * 8),
               ks_umma_desc_sw128(v_addr + kk * 2048, kBox, 1024), idesc, accumulate || kk > 0);
}

__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd1_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, uint16_t *__restrict__ out, int nq, int nk,
                   float scale_log2, int causal, KsWait wait) {
  using L = Fa1Layout;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ks_smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::bar_off);
  uint64_t *q_full = bars;
  uint64_t *k_full = bars + 1;
  uint64_t *k_empty = k_full + kStages;
  uint64_t *v_full = k_empty + kStages;
  uint64_t *v_empty = v_full + kStages;
  uint64_t *s_full = v_empty + kStages;
  uint64_t *p_full = s_full + 2;
  uint64_t *pv_done = p_full + 1;
  uint64_t *o_full = pv_done + 1;
  uint64_t *red_bar = o_full + 1;
  uint64_t *drain = red_bar + 1;
  float *red = reinterpret_cast<float *>(smem + L::red_off);
  float *lsum = reinterpret_cast<float *>(smem + L::lsum_off);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::misc_off);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + L::misc_off + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_qb = (nq + kTile - 1) / kTile;
  const int qb = num_qb - 1 - int(blockIdx.x);  // heaviest causal blocks first
  const int bh = blockIdx.y;
  const int q0 = qb * kTile;
  int n_kv = (nk + kTile - 1) / kTile;
  if (causal) n_kv = min(n_kv, (min(q0 + kTile, nq) - 1) / kTile + 1);

  if (threadIdx.x == 0) {
    ks_mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      ks_mbar_init(k_full + s, 1);
      ks_mbar_init(k_empty + s, 1);
      ks_mbar_init(v_full + s, 1);
      ks_mbar_init(v_empty + s, 1);
    }
    ks_mbar_init(s_full + 0, 1);
    ks_mbar_init(s_full + 1, 1);
    ks_mbar_init(p_full, 8);
    ks_mbar_init(pv_done, 1);
    ks_mbar_init(o_full, 1);
    ks_mbar_init(red_bar, 8);
    ks_mbar_init(drain, 1);
    *abort = 0;
    ks_fence_mbar_init();
    ks_prefetch_tmap(&tm_q);
    ks_prefetch_tmap(&tm_k);
    ks_prefetch_tmap(&tm_v);
  }
  if (warp == 9) {
    ks_tmem_alloc(tmem_slot, 512);
    ks_tmem_relinquish();
  }
  ks_tc_fence_before();
  __syncthreads();
  ks_tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      ks_mbar_arrive_expect_tx(q_full, kTileBytes);
      for (int h = 0; h < 2; ++h) ks_tma_load_3d(smem + L::q_off + h * kBox, &tm_q, q_full, h * 64, q0, bh);
      uint32_t k_armed = 0, k_par = 0, v_armed = 0, v_par = 0;
      auto load = [&](const CUtensorMap *m, uint64_t *full, uint64_t *empty, uint32_t off, int j, uint32_t &armed,
                      uint32_t &par) {
        const int st = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        if (!ks_mbar_wait(empty + st, ph ^ 1u, abort, wait)) return false;
        uint8_t *dst = smem + off + st * kTileBytes;
        ks_mbar_arrive_expect_tx(full + st, kTileBytes);
        for (int h = 0; h < 2; ++h) ks_tma_load_3d(dst + h * kBox, m, full + st, h * 64, j * kTile, bh);
        armed |= 1u << st;
        par = (par & ~(1u << st)) | (ph << st);
        return true;
      };
      bool ok = load(&tm_k, k_full, k_empty, L::k_off, 0, k_armed, k_par);
      if (ok && n_kv > 1) ok = load(&tm_k, k_full, k_empty, L::k_off, 1, k_armed, k_par);
      for (int j = 0; j < n_kv && ok; ++j) {
        ok = load(&tm_v, v_full, v_empty, L::v_off, j, v_armed, v_par);
        if (ok && j + 2 < n_kv) ok = load(&tm_k, k_full, k_empty, L::k_off, j + 2, k_armed, k_par);
      }
      // teardown: the loads issued above have landed
      ks_mbar_wait(q_full, 0, nullptr, wait);
      for (int s = 0; s < kStages; ++s) {
        if (k_armed & (1u << s)) ks_mbar_wait(k_full + s, (k_par >> s) & 1u, nullptr, wait);
        if (v_armed & (1u << s)) ks_mbar_wait(v_full + s, (v_par >> s) & 1u, nullptr, wait);
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      const uint32_t q_addr = ks_smem_u32(smem + L::q_off);
      const uint32_t k_addr = ks_smem_u32(smem + L::k_off);
      const uint32_t v_addr = ks_smem_u32(smem + L::v_off);
      const uint32_t t_o = tmem + 256;
      auto s_mma = [&](int j) {
        const int st = j % kStages;
        if (!ks_mbar_wait(k_full + st, (j / kStages) & 1, abort, wait)) return false;
        ks_tc_fence_after();
        issue_s(tmem + (j & 1) * 128, q_addr, k_addr + st * kTileBytes);
        ks_umma_commit(k_empty + st);
        ks_umma_commit(s_full + (j & 1));
        return true;
      };
      bool ok = ks_mbar_wait(q_full, 0, abort, wait) && s_mma(0);
      if (ok && n_kv > 1) ok = s_mma(1);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % kStages;
        if (!ks_mbar_wait(v_full + st, (j / kStages) & 1, abort, wait)) break;
        if (!ks_mbar_wait(p_full, j & 1, abort, wait)) break;
        ks_tc_fence_after();
        issue_pv_split(t_o, tmem + (j & 1) * 128, v_addr + st * kTileBytes, j > 0);
        ks_umma_commit(pv_done);
        ks_umma_commit(v_empty + st);
        if (j + 1 == n_kv) ks_umma_commit(o_full);
        if (j + 2 < n_kv && !s_mma(j + 2)) break;
      }
      ks_umma_commit(drain);
      ks_mbar_wait(drain, 0, nullptr, wait);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int wg = warp >> 2;        // column half of each S tile: keys [64 wg, 64 wg + 64)
    const int qd = warp & 3;         // TMEM lane quadrant
    const int row = qd * 32 + lane;  // row within the tile = TMEM lane
    const int qrow = q0 + row;
    const uint32_t lane_addr = tmem + (uint32_t(qd * 32) << 16);
    const uint32_t my_col = 64 * wg;
    const uint32_t o_col = 256 + 64 * wg;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const uint32_t s_col = (j & 1) * 128 + my_col;
      if (!ks_mbar_wait(s_full + (j & 1), (j >> 1) & 1, abort, wait)) {
        ok = false;
        break;
      }
      ks_tc_fence_after();
      uint32_t r[64];
      ks_tmem_ld32_at<0>(lane_addr + s_col, r);
      ks_tmem_ld32_at<32>(lane_addr + s_col + 32, r);
      ks_tmem_wait_ld();
      const int key0 = j * kTile + int(my_col);
      int lim = nk - key0;  // valid keys among this warpgroup's 64
      if (causal) lim = min(lim, qrow - key0 + 1);
      if (!__all_sync(0xffffffffu, lim >= 64)) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (c >= lim) r[c] = 0xff800000u;  // -inf
      }
      float mm[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        mm[u] = max3(__uint_as_float(r[u]), __uint_as_float(r[u + 4]), __uint_as_float(r[u + 8]));
#pragma unroll
      for (int c = 12; c < 60; c += 8)
#pragma unroll
        for (int u = 0; u < 4; ++u) mm[u] = max3(mm[u], __uint_as_float(r[c + u]), __uint_as_float(r[c + 4 + u]));
#pragma unroll
      for (int u = 0; u < 4; ++u) mm[u] = fmaxf(mm[u], __uint_as_float(r[60 + u]));
      const float pm = fmaxf(fmaxf(mm[0], mm[1]), fmaxf(mm[2], mm[3]));
      // exchange the partial maxima with the other warpgroup (bounded wait)
      red[((j & 1) * 2 + wg) * 128 + row] = pm;
      __syncwarp();
      if (lane == 0) ks_mbar_arrive(red_bar);
      if (!ks_mbar_wait(red_bar, j & 1, abort, wait)) {
        ok = false;
        break;
      }
      const float mx = fmaxf(pm, red[((j & 1) * 2 + (wg ^ 1)) * 128 + row]);
      const float m_new = fmaxf(m, mx * scale_log2);
      const bool grow = m_new > m + 8.f;  // also true on the first finite max
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        // O must hold every earlier P V before it is rescaled
        if (!ks_mbar_wait(pv_done, (j - 1) & 1, abort, wait)) {
          ok = false;
          break;
        }
        ks_tc_fence_after();
        const float alpha = grow ? ex2(m - m_new) : 1.f;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          ks_tmem_ld32(lane_addr + o_col + c * 32, o);
          ks_tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(lane_addr + o_col + c * 32, o);
        }
        ks_tmem_wait_st();
      }
      if (grow) {
        l *= ex2(m - m_new);
        m = m_new;
      }
      const float neg_m = (m == -INFINITY) ? 0.f : -m;
      F2 rsum[4] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
      const F2 sc2{scale_log2, scale_log2}, nm2{neg_m, neg_m};
      uint32_t p[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const F2 x = fma2(F2{__uint_as_float(r[2 * c]), __uint_as_float(r[2 * c + 1])}, sc2, nm2);
        const F2 e{ex2(x.x), ex2(x.y)};
        rsum[c & 3] = add2(rsum[c & 3], e);
        p[c] = ks_pack_bf16x2(e.x, e.y);
      }
      ks_tmem_st32_at<0>(lane_addr + s_col, p);
      const F2 rs2 = add2(add2(rsum[0], rsum[1]), add2(rsum[2], rsum[3]));
      l += rs2.x + rs2.y;
      ks_tmem_wait_st();
      ks_tc_fence_before();
      __syncwarp();
      if (lane == 0) ks_mbar_arrive(p_full);
    }
    // epilogue: row sum = both warpgroups' partial sums; O / l -> bf16
    if (ok) {
      lsum[wg * 128 + row] = l;
      __syncwarp();
      if (lane == 0) ks_mbar_arrive(red_bar);
      ok = ks_mbar_wait(red_bar, n_kv & 1, abort, wait) && ks_mbar_wait(o_full, 0, abort, wait);
    }
    if (ok) {
      ks_tc_fence_after();
      const float lt = l + lsum[(wg ^ 1) * 128 + row];
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      uint16_t *dst = out + (int64_t(bh) * nq + qrow) * kD + my_col;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        ks_tmem_ld32(lane_addr + o_col + c * 32, o);
        ks_tmem_wait_ld();
        if (qrow < nq) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = ks_pack_bf16x2(__uint_as_float(o[v * 8 + 0]) * inv, __uint_as_float(o[v * 8 + 1]) * inv);
            w.y = ks_pack_bf16x2(__uint_as_float(o[v * 8 + 2]) * inv, __uint_as_float(o[v * 8 + 3]) * inv);
            w.z = ks_pack_bf16x2(__uint_as_float(o[v * 8 + 4]) * inv, __uint_as_float(o[v * 8 + 5]) * inv);
            w.w = ks_pack_bf16x2(__uint_as_float(o[v * 8 + 6]) * inv, __uint_as_float(o[v * 8 + 7]) * inv);
            *reinterpret_cast<uint4 *>(dst + c * 32 + v * 8) = w;
          }
        }
      }
    }
  }

  ks_tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    ks_tc_fence_after();
    ks_tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// CUDA-core path for head dims other than 128 (d <= 256; the reference's gate
// shapes use d = 16 and 32): one warp per query row, keys in chunks of 32
// (one key per lane for the scores), online softmax with warp shuffles, each
// lane accumulating d/32 output columns.
// ---------------------------------------------------------------------------
constexpr int kSimtMaxD = 256;

__global__ void __launch_bounds__(128) fa_simt_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k,
                                                      const uint16_t *__restrict__ v, uint16_t *__restrict__ out,
                                                      int nq, int nk, int d, float scale_log2, int causal) {
  __shared__ float qs[4][kSimtMaxD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + warp;
  const int64_t bh = blockIdx.y;
  if (row >= nq) return;
  const uint16_t *qr = q + (bh * nq + row) * d;
  for (int c = lane; c < d; c += 32) qs[warp][c] = ks_bf16_to_f32(qr[c]);
  __syncwarp();
  const uint16_t *kb = k + bh * nk * d;
  const uint16_t *vb = v + bh * nk * d;
  const int kend = causal ? min(nk, row + 1) : nk;
  float m = -INFINITY, l = 0.f;
  float o[kSimtMaxD / 32];
#pragma unroll
  for (int i = 0; i < kSimtMaxD / 32; ++i) o[i] = 0.f;
  for (int k0 = 0; k0 < kend; k0 += 32) {
    const int key = k0 + lane;
    float s = -INFINITY;
    if (key < kend) {
      const uint16_t *kr = kb + int64_t(key) * d;
      float acc = 0.f;
      for (int c = 0; c < d; ++c) acc = fmaf(qs[warp][c], ks_bf16_to_f32(kr[c]), acc);
      s = acc * scale_log2;
    }
    const float mx = ks_warp_max(s);
    const float m_new = fmaxf(m, mx);
    const float alpha = ex2(m - m_new);
    const float p = (key < kend) ? ex2(s - m_new) : 0.f;
    l = l * alpha + ks_warp_sum(p);
#pragma unroll
    for (int i = 0; i < kSimtMaxD / 32; ++i) o[i] *= alpha;
    const int nkeys = min(32, kend - k0);
    for (int t = 0; t < nkeys; ++t) {
      const float pt = __shfl_sync(0xffffffffu, p, t);
      const uint16_t *vr = vb + int64_t(k0 + t) * d;
#pragma unroll
      for (int i = 0; i < kSimtMaxD / 32; ++i) {
        const int c = lane + 32 * i;
        if (c < d) o[i] = fmaf(pt, ks_bf16_to_f32(vr[c]), o[i]);
      }
    }
    m = m_new;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  uint16_t *orow = out + (bh * nq + row) * d;
#pragma unroll
  for (int i = 0; i < kSimtMaxD / 32; ++i) {
    const int c = lane + 32 * i;
    if (c < d) orow[c] = ks_f32_to_bf16(o[i] * inv);
  }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int D>
int launch_fwd(unsigned grid, cudaStream_t st, const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv,
               const ks_flash_attention_args &a, uint64_t bh, float scale_log2, int causal, bool ring) {
  cudaError_t e;
  if (ring) {
    e = cudaFuncSetAttribute(fa_ring_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(FaRingLayout<D>::smem_request));
    if (e != cudaSuccess) return ks::map_cuda(e);
    fa_ring_kernel<D><<<grid, kThreads2, FaRingLayout<D>::smem_request, st>>>(
        tq, tk, tv, static_cast<uint16_t *>(a.out), int(a.nq), int(a.nk), int(bh), scale_log2, causal,
        ks::wait_ctx());
    return ks::map_cuda(cudaGetLastError());
  }
  // O: [32 columns x 32 rows] boxes per head, 64-byte swizzle (the epilogue's staging layout)
  CUtensorMap to;
  const uint64_t d = uint64_t(D), rs = d * 2;
  int s = ks::encode_tmap_3d(&to, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a.out, d, uint64_t(a.nq), bh, rs,
                             rs * uint64_t(a.nq), 32, 32, 1, CU_TENSOR_MAP_SWIZZLE_64B);
  if (s != KS_OK) return s;
  e = cudaFuncSetAttribute(fa_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           int(FaLayout<D>::smem_request));
  if (e != cudaSuccess) return ks::map_cuda(e);
  fa_fwd_kernel<D><<<grid, kThreads2, FaLayout<D>::smem_request, st>>>(tq, tk, tv, to, int(a.nq), int(a.nk),
                                                                       int(bh), scale_log2, causal, ks::wait_ctx());
  return ks::map_cuda(cudaGetLastError());
}

}  // namespace

extern "C" {

int ks_flash_attention_validate(const ks_flash_attention_config *cfg, const ks_flash_attention_args *a,
                                char *reason, size_t len) {
  if (!cfg || !a) return KS_ERR_INVALID_ARGS;
  if ((cfg->tile_m != 128 && cfg->tile_m != 256) ||
      (cfg->tile_n != 128 && !(cfg->tile_n == 64 && cfg->tile_m == 256))) {
    ks::set_reason(reason, len,
                   "flash_attention: tile_m must be 128 or 256 (query rows per CTA: one or two UMMA M=128 "
                   "tiles) and tile_n 128 (keys per softmax step), or 64 with tile_m 256 (S in 64-key slots)");
    return KS_ERR_INVALID_CONFIG;
  }
  if (cfg->stages != 2) {
    ks::set_reason(reason, len, "flash_attention: stages must be 2 (K/V ring depth)");
    return KS_ERR_INVALID_CONFIG;
  }
  if (cfg->causal != 0 && cfg->causal != 1) {
    ks::set_reason(reason, len, "flash_attention: causal must be 0 or 1");
    return KS_ERR_INVALID_CONFIG;
  }
  if (a->d < 1 || a->d > kSimtMaxD) {
    ks::set_reason(reason, len, "flash_attention: head dim %lld unsupported (1..256; tensor cores at d = 128, and at d = 64 with tile_m 256)",
                   (long long)a->d);
    return KS_ERR_INVALID_CONFIG;
  }
  if (a->batch <= 0 || a->heads <= 0 || a->nq <= 0 || a->nk <= 0) {
    ks::set_reason(reason, len, "flash_attention: batch, heads, nq, nk must be positive");
    return KS_ERR_INVALID_ARGS;
  }
  if (a->batch * a->heads > 65535 || a->nq >= (1LL << 31) || a->nk >= (1LL << 31)) {
    ks::set_reason(reason, len, "flash_attention: batch*heads <= 65535 and sequence lengths < 2^31");
    return KS_ERR_INVALID_ARGS;
  }
  ks::set_reason(reason, len, "");
  return KS_OK;
}

int ks_flash_attention_launch(const ks_flash_attention_config *cfg, const ks_flash_attention_args *a,
                              void *stream) {
  int s = ks_flash_attention_validate(cfg, a, nullptr, 0);
  if (s != KS_OK) return s;
  if (!a->q || !a->k || !a->v || !a->out) return KS_ERR_INVALID_ARGS;
  if ((s = ks::check_arch_sm100()) != KS_OK) return s;
  const uint64_t bh = uint64_t(a->batch * a->heads);
  const float scale = a->scale > 0.f ? a->scale : 1.f / sqrtf(float(a->d));
  const float scale_log2 = scale * 1.4426950408889634f;
  // tensor cores: d = 128 with either config, d = 64 with two query tiles per CTA
  const bool tc_d = a->d == kD || (a->d == 64 && cfg->tile_m == 256);
  if (!tc_d || !aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out)) {
    dim3 grid(unsigned((a->nq + 3) / 4), unsigned(bh));
    fa_simt_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t *>(a->q), static_cast<const uint16_t *>(a->k),
        static_cast<const uint16_t *>(a->v), static_cast<uint16_t *>(a->out), int(a->nq), int(a->nk), int(a->d),
        scale_log2, cfg->causal);
    return ks::map_cuda(cudaGetLastError());
  }
  CUtensorMap tq, tk, tv;
  const uint64_t d = uint64_t(a->d), rs = d * 2;
  s = ks::encode_tmap_3d(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a->q, d, uint64_t(a->nq), bh, rs,
                         rs * uint64_t(a->nq), 64, 128, 1, CU_TENSOR_MAP_SWIZZLE_128B);
  if (s == KS_OK)
    s = ks::encode_tmap_3d(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a->k, d, uint64_t(a->nk), bh, rs,
                           rs * uint64_t(a->nk), 64, 128, 1, CU_TENSOR_MAP_SWIZZLE_128B);
  if (s == KS_OK)
    s = ks::encode_tmap_3d(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a->v, d, uint64_t(a->nk), bh, rs,
                           rs * uint64_t(a->nk), 64, 128, 1, CU_TENSOR_MAP_SWIZZLE_128B);
  if (s != KS_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cfg->tile_m == 128) {
    cudaError_t e = cudaFuncSetAttribute(fa_fwd1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(Fa1Layout::smem_request));
    if (e != cudaSuccess) return ks::map_cuda(e);
    dim3 grid(unsigned((a->nq + kTile - 1) / kTile), unsigned(bh));
    fa_fwd1_kernel<<<grid, kThreads, Fa1Layout::smem_request, st>>>(
        tq, tk, tv, static_cast<uint16_t *>(a->out), int(a->nq), int(a->nk), scale_log2, cfg->causal,
        ks::wait_ctx());
    return ks::map_cuda(cudaGetLastError());
  }
  // persistent: one CTA per SM (fewer when there are fewer work items)
  const int64_t items = ((a->nq + 2 * kTile - 1) / (2 * kTile)) * int64_t(bh);
  const int sms = ks::sm_count();
  const unsigned grid = unsigned(items < sms ? items : sms);
  const bool ring = cfg->tile_n == 64;
  return a->d == kD ? launch_fwd<kD>(grid, st, tq, tk, tv, *a, bh, scale_log2, cfg->causal, ring)
                    : launch_fwd<64>(grid, st, tq, tk, tv, *a, bh, scale_log2, cfg->causal, ring);
}

}  // extern "C"
