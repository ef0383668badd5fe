// Windowed causal prefill for sm_100a: warp-specialised tcgen05 / TMEM kernel.
//
// One CTA owns two 128-row query tiles (Q0, Q1) of one (batch, q head) and
// streams 128-key K/V tiles over its causal range:
//
//   warp 8       TMA producer. Q once (8 levels x 2 halves per tile); per key
//                tile only the in-window K levels (L = D_eff/16 of the nearer
//                query tile) and the two 64-dim V boxes.
//   warp 9       MMA issuer and TMEM owner (512 columns). S_t is computed
//                over L(t, j) K-steps of 16 dims. P_t (bf16) goes into columns
//                64..127 of the OTHER tile's S (free once that tile has read its
//                scores into registers) and is read by O_t += P_t V from TMEM. So
//                S_t(j+1) does not wait for P_t(j): per key tile j the warp issues
//                O_0 += P_0(j) V_j, S_1(j+1), O_1 += P_1(j) V_j, S_0(j+2), and a
//                softmax warp finds its next scores ready when it finishes a step.
//   warps 0-3/4-7  softmax for Q0 / Q1: one query row per thread, online
//                softmax in the log2 domain, lazy O rescale, epilogue.
//
// Issue discipline: the producer and MMA warps run their schedules with all 32
// lanes and warp-uniform operands (TMEM base broadcast, descriptors built once
// and advanced by adds); one elected lane issues each TMA / tcgen05.mma /
// tcgen05.commit. 128-column MMAs issued this way run at the tensor pipe's
// peak; a lane-0-only branch costs several times more per instruction.
//
// The window is the reference's tile quantisation (atflash/reference.py:59-68,
// atflash/window_table.py:70-76) at block_m = block_n = 128: for query tile q0
// and key tile n0 the QK contraction runs over D_eff(z_min) dims with
// z_min = max(0, q0 - (n0+127)); D_eff(z) = 16 * #{i : zhi[i] >= z}
// (window_tables/atflash_window.py:85-108). The causal diagonal and ragged
// tails use per-element predicates.
//
// Shared memory (1024-aligned):
//   Q  2 tiles x 8 level slabs x 4 KB. A slab is the canonical no-swizzle
//      K-major layout: two halves (dims 0-7 and 8-15 of the level), each
//      128 rows x 16 B, so core matrices (8 rows x 16 B) are contiguous:
//      LBO (K direction) = 2 KB, SBO (8-row groups) = 128 B.
//   K  2 stages x 8 slabs x 4 KB, one slab per in-window level; only the L
//      in-window levels are loaded. sorted-pair: one 5-d box {16 dims, 128
//      keys, L levels} per key tile (level i is dims 16i..16i+15), slabs of
//      128 keys x 32 B with 32-byte swizzle, K-major (SBO = 256 B).
//      rotate_half: two 8-dim boxes per level (chunks 7-i and 15-i), in the Q
//      slab layout.
//   V  2 stages x 2 boxes (dims 0-63, 64-127) x 128 keys x 128 B, 128B swizzle;
//      the PV B operand is MN-major: LBO (next 64 dims) = 16 KB, SBO (next 8
//      keys) = 1 KB.
// TMEM columns: S_t at 128t, O_t at 256 + 128t; P_t at 128(1-t) + 64.
#include <math.h>

#include "atf_internal.h"
#include "atf_ptx.cuh"
#include "rope_math.cuh"

namespace atf {
namespace prefill {

// MMA groups are issued from one asm block each, under a single elect: the MMA
// warp shares its sub-partition with two softmax warps, so fewer instructions
// per tcgen05.mma keep the tensor pipe fed.
//
// one elected lane issues the 8 PV MMAs (K = 128 keys) of a tile and the commit
__device__ __forceinline__ void pv_group_asm(uint32_t o_tmem, uint32_t p_tmem, uint64_t vd, uint32_t idesc,
                                             uint32_t acc0, uint32_t bar_addr) {
  asm volatile(
      "{\n\t.reg .pred pe, pa;\n\t.reg .b64 b;\n\t.reg .b32 a;\n\t"
      "elect.sync _|pe, 0xffffffff;\n\t"
      "setp.ne.b32 pa, %4, 0;\n\t"
      "@pe tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, pa;\n\t"
      "add.u32 a, %1, 8;\n\tadd.u64 b, %2, 128;\n\t"
      "@pe tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, 1;\n\t"
      "add.u32 a, a, 8;\n\tadd.u64 b, b, 128;\n\t"
      "@pe tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, 1;\n\t"
      "add.u32 a, a, 8;\n\tadd.u64 b, b, 128;\n\t"
      "@pe tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, 1;\n\t"
      "add.u32 a, a, 8;\n\tadd.u64 b, b, 128;\n\t"
      "@pe tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, 1;\n\t"
      "add.u32 a, a, 8;\n\tadd.u64 b, b, 128;\n\t"
      "@pe tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, 1;\n\t"
      "add.u32 a, a, 8;\n\tadd.u64 b, b, 128;\n\t"
      "@pe tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, 1;\n\t"
      "add.u32 a, a, 8;\n\tadd.u64 b, b, 128;\n\t"
      "@pe tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, 1;\n\t"
      "@pe tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%5];\n\t}"
      ::"r"(o_tmem), "r"(p_tmem), "l"(vd), "r"(idesc), "r"(acc0), "r"(bar_addr)
      : "memory");
}
// one elected lane issues the L (1..8) QK MMAs of a tile and the commit; level
// i advances A and B by one 4 KB slab (descriptor start field += 256)
__device__ __forceinline__ void qk_group_asm(uint32_t d_tmem, uint64_t qd, uint64_t kd, uint32_t idesc, int L,
                                             uint32_t bar_addr) {
  asm volatile(
      "{\n\t.reg .pred pe, p1, p2, p3, p4, p5, p6, p7;\n\t.reg .b64 a, b;\n\t"
      "elect.sync _|pe, 0xffffffff;\n\t"
      "setp.gt.and.s32 p1, %4, 1, pe;\n\tsetp.gt.and.s32 p2, %4, 2, pe;\n\tsetp.gt.and.s32 p3, %4, 3, pe;\n\t"
      "setp.gt.and.s32 p4, %4, 4, pe;\n\tsetp.gt.and.s32 p5, %4, 5, pe;\n\tsetp.gt.and.s32 p6, %4, 6, pe;\n\t"
      "setp.gt.and.s32 p7, %4, 7, pe;\n\t"
      "@pe tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, 0;\n\t"
      "add.u64 a, %1, 256;\n\tadd.u64 b, %2, 256;\n\t"
      "@p1 tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, 1;\n\t"
      "add.u64 a, a, 256;\n\tadd.u64 b, b, 256;\n\t"
      "@p2 tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, 1;\n\t"
      "add.u64 a, a, 256;\n\tadd.u64 b, b, 256;\n\t"
      "@p3 tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, 1;\n\t"
      "add.u64 a, a, 256;\n\tadd.u64 b, b, 256;\n\t"
      "@p4 tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, 1;\n\t"
      "add.u64 a, a, 256;\n\tadd.u64 b, b, 256;\n\t"
      "@p5 tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, 1;\n\t"
      "add.u64 a, a, 256;\n\tadd.u64 b, b, 256;\n\t"
      "@p6 tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, 1;\n\t"
      "add.u64 a, a, 256;\n\tadd.u64 b, b, 256;\n\t"
      "@p7 tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, 1;\n\t"
      "@pe tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%5];\n\t}"
      ::"r"(d_tmem), "l"(qd), "l"(kd), "r"(idesc), "r"(L), "r"(bar_addr)
      : "memory");
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

constexpr int BM = 128, BN = 128, HD = 128, NQ = 2, KST = 2, VST = 2;
// Warps 10 and 11 have no role: they complete the third warpgroup so that the
// register split below (setmaxnreg acts on whole warpgroups) can take
// registers from the producer / MMA group and give them to the softmax groups.
constexpr int WARP_LOAD = 8, WARP_MMA = 9, NUM_WARPS = 12, THREADS = NUM_WARPS * 32;
// Registers per thread after the split. The block launches with THREADS x the
// compiled count (168 under __launch_bounds__(THREADS, 1)); the host refuses to
// launch unless 128 x REG_SMALL + 256 x REG_SOFTMAX fits in that.
constexpr int REG_SMALL = 80, REG_SOFTMAX = 208;
constexpr long long REG_SPLIT_TOTAL = 128LL * REG_SMALL + 256LL * REG_SOFTMAX;
template <int N>
__device__ __forceinline__ void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
constexpr uint32_t QHALF_BYTES = BM * 16;             // 2 KB
constexpr uint32_t QSLAB_BYTES = 2 * QHALF_BYTES;     // 4 KB
constexpr uint32_t QTILE_BYTES = 8 * QSLAB_BYTES;     // 32 KB
constexpr uint32_t KHALF_BYTES = BN * 16;             // 2 KB
constexpr uint32_t KSLAB_BYTES = 2 * KHALF_BYTES;     // 4 KB
constexpr uint32_t KSTAGE_BYTES = 8 * KSLAB_BYTES;    // 32 KB
// sorted-pair K tensor maps over (16 dims of a level, key, level, kv head,
// batch); map L-1 moves the box {16, 128, L}: exactly the L in-window levels,
// as [L][128 keys][32 B] with 32-byte swizzle
struct KLevelMaps {
  CUtensorMap lv[ATF_MAX_LEVELS];
};
constexpr uint32_t VBOX_BYTES = BN * 128;             // 16 KB
constexpr uint32_t VSTAGE_BYTES = 2 * VBOX_BYTES;     // 32 KB
constexpr uint32_t OFF_Q = 0;
constexpr uint32_t OFF_K = OFF_Q + NQ * QTILE_BYTES;
constexpr uint32_t OFF_V = OFF_K + KST * KSTAGE_BYTES;
constexpr uint32_t OFF_BAR = OFF_V + VST * VSTAGE_BYTES;

enum {
  B_Q = 0,
  B_KFULL = 1,
  B_KEMPTY = B_KFULL + KST,
  B_VFULL = B_KEMPTY + KST,
  B_VEMPTY = B_VFULL + VST,
  B_SFULL = B_VEMPTY + VST,   // [t]
  B_PFULL = B_SFULL + NQ,     // [t]
  B_ODONE = B_PFULL + NQ,     // [t], one phase per O += P V
  B_OFINAL = B_ODONE + NQ,    // [t], single phase: the tile's last O += P V done
  B_LOADED = B_OFINAL + NQ,   // [t], phase j: tile t's softmax has read S_t(j) into registers
  B_FINAL = B_LOADED + NQ,
  NUM_BARS
};
constexpr uint32_t OFF_ABORT = OFF_BAR + 8 * NUM_BARS;
constexpr uint32_t OFF_TMEM = OFF_ABORT + 16;
constexpr uint32_t SMEM_USED = OFF_TMEM + 16;
constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;  // slack for 1024-B alignment

constexpr uint32_t IDESC_QK = make_idesc_bf16(128, BN, 0, 0);
constexpr uint32_t IDESC_PV = make_idesc_bf16(128, HD, 0, 1);
constexpr uint32_t FULL = 0xffffffffu;

struct Args {
  int B, Sq, Sk, Hq, G, n_qblk;
  // query row ranges: range r covers rows [r_lo[r], r_hi[r]) in r_nblk[r] blocks
  // of BM * NQ rows; n_qblk is their sum
  int nrange;
  int r_lo[2], r_hi[2], r_nblk[2];
  long long q_offset;
  float scale_log2;
  int causal, layout, window;
  int zhi[ATF_MAX_LEVELS];
  __nv_bfloat16* out;
  long long o_sb, o_ss, o_sh;
  float* lse;
  int* err;
  // RoPE of q at load (qrot): the pre-RoPE rows and the fp32 cos / sin tables
  int qrot;
  const __nv_bfloat16* q;
  long long q_sb, q_ss, q_sh;
  const float* qcos;
  const float* qsin;
  long long cs_stride;
};

// The window of one query tile (rows row0..row0+127) as key-tile limits, set
// once per CTA and held in registers: key tile j reads level i when
// j >= lim[i]. The tile's smallest distance is z_min(j) = max(0, q_offset + row0
// - (128 j + 127)), and level i is read when z_min(j) <= zhi[i] (level 0
// always: zhi[0] covers every distance), i.e. from
// j = ceil((q_offset + row0 - 127 - zhi[i]) / 128) on.
__device__ __forceinline__ void window_limits(const Args& a, int row0, int (&lim)[ATF_MAX_LEVELS]) {
  const long long base = a.q_offset + row0 - (BN - 1);
#pragma unroll
  for (int i = 0; i < ATF_MAX_LEVELS; ++i) {
    const long long x = base - a.zhi[i];
    long long j = (!a.window || i == 0 || x <= 0) ? 0 : (x + BN - 1) / BN;
    lim[i] = static_cast<int>(j > 0x7fffffffLL ? 0x7fffffffLL : j);
  }
}
// levels of key tile j: the L (1..8) in-window 16-dim levels of the pair
__device__ __forceinline__ int levels_for(const int (&lim)[ATF_MAX_LEVELS], int j) {
  int L = 0;
#pragma unroll
  for (int i = 0; i < ATF_MAX_LEVELS; ++i) L += j >= lim[i] ? 1 : 0;
  return L;
}
// first key tile that needs per-element masks: a key past the query row
// (causal) or past the end of the keys
__device__ __forceinline__ int first_masked_tile(const Args& a, int row0) {
  long long jm = a.Sk / BN;  // 128 j + 127 >= Sk from j = ceil((Sk - 127) / 128) = floor(Sk / 128)
  if (a.causal) {
    const long long x = a.q_offset + row0 - (BN - 1);  // 128 j > x for a masked tile
    const long long jc = x < 0 ? 0 : x / BN + 1;
    if (jc < jm) jm = jc;
  }
  return static_cast<int>(jm > 0x7fffffffLL ? 0x7fffffffLL : jm);
}

// Column of the first element of half `hh` of level `i` along head_dim.
// sorted-pair order: level i = dims [16i, 16i+16).
// rotate_half order (HF): sorted pairs 8i..8i+7 are HF dims [56-8i, 64-8i) and
// [120-8i, 128-8i).
__device__ __forceinline__ int level_col(int layout, int i, int hh) {
  return layout == ATF_LAYOUT_SORTED_PAIR ? 16 * i + 8 * hh : 64 * hh + 8 * (7 - i);
}

// Waits with no abort short-cut: used to drain this CTA's own asynchronous
// copies / MMAs before the CTA's shared memory or TMEM is released.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
}

__global__ void __launch_bounds__(THREADS, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ KLevelMaps tmKL,
                   const __grid_constant__ CUtensorMap tmV, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t sb = (raw_u32 + 1023u) & ~1023u;
  uint8_t* sp = smem_raw + (sb - raw_u32);
  volatile int* s_abort = reinterpret_cast<volatile int*>(sp + OFF_ABORT);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sp + OFF_TMEM);
  auto bar = [&](int i) -> uint32_t { return sb + OFF_BAR + 8u * static_cast<uint32_t>(i); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Work unit order: one (batch, kv head) group at a time, longest query
  // blocks first inside it, the G query heads of the group adjacent. The CTAs
  // resident together then read a single kv head's K/V, whose causal range
  // (256 B x 2 per key) stays in L2, so HBM sees each K/V byte about once.
  const int Hkv = a.Hq / a.G;
  const int per_group = a.n_qblk * a.G;
  const int grp = static_cast<int>(blockIdx.x) / per_group;
  const int rem = static_cast<int>(blockIdx.x) % per_group;
  // blocks of the later row range first, each range's blocks latest rows first
  const int qidx = a.n_qblk - 1 - rem / a.G;
  const int rng = (a.nrange > 1 && qidx >= a.r_nblk[0]) ? 1 : 0;
  const int row_base = a.r_lo[rng] + (qidx - (rng ? a.r_nblk[0] : 0)) * (BM * NQ);
  const int row_end = rng ? a.r_hi[1] : a.r_hi[0];
  const int bi = grp / Hkv;
  const int hk = grp % Hkv;
  const int h = hk * a.G + rem % a.G;
  int row0[NQ], nk[NQ];
#pragma unroll
  for (int t = 0; t < NQ; ++t) {
    row0[t] = row_base + t * BM;
    if (row0[t] >= row_end) {
      nk[t] = 0;
    } else {
      long long kend = a.causal ? a.q_offset + row0[t] + BM : a.Sk;
      if (kend > a.Sk) kend = a.Sk;
      nk[t] = kend > 0 ? static_cast<int>((kend + BN - 1) / BN) : 0;
    }
  }
  const int nk_max = nk[0] > nk[1] ? nk[0] : nk[1];
  int lim[NQ][ATF_MAX_LEVELS];
#pragma unroll
  for (int t = 0; t < NQ; ++t) window_limits(a, row0[t], lim[t]);

  if (threadIdx.x == 0) {
    *s_abort = (a.err != nullptr && *reinterpret_cast<volatile int*>(a.err) != 0) ? 1 : 0;
    // Q arrives by TMA (one expect_tx arrival), or rotated by the softmax threads
    mbar_init(bar(B_Q), a.qrot ? NQ * 128 : 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(bar(B_KFULL + s), 1);
      mbar_init(bar(B_KEMPTY + s), 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(bar(B_VFULL + s), 1);
      mbar_init(bar(B_VEMPTY + s), 1);
    }
    for (int t = 0; t < NQ; ++t) {
      mbar_init(bar(B_SFULL + t), 1);
      mbar_init(bar(B_PFULL + t), 128);
      mbar_init(bar(B_ODONE + t), 1);
      mbar_init(bar(B_OFINAL + t), 1);
      mbar_init(bar(B_LOADED + t), 128);
    }
    mbar_init(bar(B_FINAL), 1);
    fence_mbar_init();
  }
  if (warp == WARP_LOAD && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    for (int L = 0; L < ATF_MAX_LEVELS; ++L) tma_prefetch_desc(&tmKL.lv[L]);
    tma_prefetch_desc(&tmV);
  }
  if (warp == WARP_MMA) {
    tmem_alloc(smem_u32(s_tmem), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const AbortCtl ab{s_abort, a.err};
  const bool start_ok = (*s_abort == 0);
  if (warp >= 8) {
    reg_dealloc<REG_SMALL>();
    if (start_ok && warp == WARP_LOAD) {
      // ---------------------------------------------------------------- producer
      // All 32 lanes run this loop with warp-uniform values; one elected lane
      // issues each TMA / expect_tx.
      int issued_k = 0, issued_v = 0;
      bool ok = true;
      if (!a.qrot) {
        uint32_t qbytes = 0;
#pragma unroll
        for (int t = 0; t < NQ; ++t) qbytes += nk[t] > 0 ? QTILE_BYTES : 0u;
        mbar_arrive_expect_tx_elect(bar(B_Q), qbytes);
#pragma unroll
        for (int t = 0; t < NQ; ++t) {
          if (nk[t] == 0) continue;
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
              tma_load_4d_elect(sb + OFF_Q + t * QTILE_BYTES + i * QSLAB_BYTES + hh * QHALF_BYTES, &tmQ,
                                bar(B_Q), level_col(a.layout, i, hh), row0[t], h, bi);
        }
      }
      for (int j = 0; j < nk_max; ++j) {
        const int ks = j % KST, vs = j % VST;
        ok = __all_sync(FULL, mbar_wait_inl(bar(B_KEMPTY + ks), ((j / KST) & 1) ^ 1, ab, kDevErrTimeout));
        if (!ok) break;
        int L = 0;
#pragma unroll
        for (int t = 0; t < NQ; ++t)
          if (j < nk[t]) {
            const int lt = levels_for(lim[t], j);
            L = lt > L ? lt : L;
          }
        const uint32_t kdst = sb + OFF_K + ks * KSTAGE_BYTES;
        if (a.layout == ATF_LAYOUT_SORTED_PAIR) {
          // one 5-d box: the L in-window levels (dims 0..16L-1), one 4 KB slab each
          mbar_arrive_expect_tx_elect(bar(B_KFULL + ks), static_cast<uint32_t>(L) * KSLAB_BYTES);
          if (elect_one_lane()) tma_load_5d(kdst, &tmKL.lv[L - 1], bar(B_KFULL + ks), 0, j * BN, 0, hk, bi);
          __syncwarp();
        } else {
          // rotate_half: a level is two 8-dim chunks 64 dims apart, one box each
          mbar_arrive_expect_tx_elect(bar(B_KFULL + ks), static_cast<uint32_t>(L) * KSLAB_BYTES);
          for (int i = 0; i < L; ++i) {
            tma_load_4d_elect(kdst + i * KSLAB_BYTES, &tmK, bar(B_KFULL + ks), level_col(a.layout, i, 0),
                              j * BN, hk, bi);
            tma_load_4d_elect(kdst + i * KSLAB_BYTES + KHALF_BYTES, &tmK, bar(B_KFULL + ks),
                              level_col(a.layout, i, 1), j * BN, hk, bi);
          }
        }
        issued_k = j + 1;
        ok = __all_sync(FULL, mbar_wait_inl(bar(B_VEMPTY + vs), ((j / VST) & 1) ^ 1, ab, kDevErrTimeout));
        if (!ok) break;
        mbar_arrive_expect_tx_elect(bar(B_VFULL + vs), VSTAGE_BYTES);
        tma_load_4d_elect(sb + OFF_V + vs * VSTAGE_BYTES, &tmV, bar(B_VFULL + vs), 0, j * BN, hk, bi);
        tma_load_4d_elect(sb + OFF_V + vs * VSTAGE_BYTES + VBOX_BYTES, &tmV, bar(B_VFULL + vs), 64,
                          j * BN, hk, bi);
        issued_v = j + 1;
      }
      // Drain: every copy this warp issued must land before shared memory is
      // released (no-op on the normal path, where the MMA warp consumed them).
      drain_wait(bar(B_Q), 0);
      for (int j = issued_k - KST; j < issued_k; ++j)
        if (j >= 0) drain_wait(bar(B_KFULL + j % KST), (j / KST) & 1);
      for (int j = issued_v - VST; j < issued_v; ++j)
        if (j >= 0) drain_wait(bar(B_VFULL + j % VST), (j / VST) & 1);
      __syncwarp();
    } else if (start_ok && warp == WARP_MMA) {
      // ---------------------------------------------------------------- MMA issuer
      // Descriptors are built once and advanced by adding (byte offset >> 4) to
      // the start-address field (all offsets stay inside the 14-bit field).
      const uint32_t tm = __shfl_sync(FULL, tmem, 0);
      const uint64_t qdesc0 = make_sdesc(sb + OFF_Q, QHALF_BYTES, 128, kLayoutNone);
      const uint64_t kdesc0 = make_sdesc(sb + OFF_K, KHALF_BYTES, 128, kLayoutNone);
      // sorted-pair K level slabs: 128 keys x 32 B, 32-byte swizzle (SBO = 8 rows)
      const uint64_t kdesc32 = make_sdesc(sb + OFF_K, 16, 256, kLayoutSw32);
      const bool sorted = a.layout == ATF_LAYOUT_SORTED_PAIR;
      const uint64_t vdesc0 = make_sdesc(sb + OFF_V, VBOX_BYTES, 1024, kLayoutSw128);
      const int nk0 = nk[0], nk1 = nk[1];
      // S_t(j) into tile t's S columns
      auto issue_S = [&](int t, int j) {
        const int L = levels_for(lim[t], j);
        const uint32_t d_tmem = tm + static_cast<uint32_t>(t * 128);
        const uint64_t qd = qdesc0 + ((t * QTILE_BYTES) >> 4);
        const uint64_t kd = (sorted ? kdesc32 : kdesc0) + (((j % KST) * KSTAGE_BYTES) >> 4);
        qk_group_asm(d_tmem, qd, kd, IDESC_QK, L, bar(B_SFULL + t));
      };
      // O_t += P_t(j) V_j; P_t sits in columns 64..127 of the other tile's S
      auto issue_PV = [&](int t, int j) {
        const uint32_t o_tmem = tm + 256u + static_cast<uint32_t>(t * 128);
        const uint32_t p_tmem = tm + static_cast<uint32_t>((1 - t) * 128 + 64);
        const uint64_t vd = vdesc0 + (((j % VST) * VSTAGE_BYTES) >> 4);
        pv_group_asm(o_tmem, p_tmem, vd, IDESC_PV, j > 0 ? 1u : 0u, bar(B_ODONE + t));
      };
      // K tiles are waited for in order, once each
      int k_waited = -1;
      auto kwait = [&](int j) -> bool {
        while (k_waited < j) {
          ++k_waited;
          if (!__all_sync(FULL, mbar_wait_inl(bar(B_KFULL + k_waited % KST), (k_waited / KST) & 1, ab,
                                          kDevErrTimeout)))
            return false;
          tc_fence_after();
        }
        return true;
      };
      auto wait_loaded = [&](int t, int j) -> bool {
        const bool w = __all_sync(FULL, mbar_wait_inl(bar(B_LOADED + t), j & 1, ab, kDevErrTimeout));
        tc_fence_after();
        return w;
      };
      // A K stage is released after the last S that reads it: S_1(j) when tile 1
      // has key tile j, else S_0(j).
      bool ok = __all_sync(FULL, mbar_wait_inl(bar(B_Q), 0, ab, kDevErrTimeout));
      tc_fence_after();
      if (ok && nk_max > 0 && (ok = kwait(0))) {
        if (nk0 > 0) issue_S(0, 0);
        if (nk1 > 0) issue_S(1, 0);
        tc_commit_elect(bar(B_KEMPTY + 0));
      }
      // S_0(1) once tile 0 has read S_0(0)
      if (ok && nk0 > 1 && (ok = kwait(1) && wait_loaded(0, 0))) {
        issue_S(0, 1);
        if (1 >= nk1) tc_commit_elect(bar(B_KEMPTY + 1 % KST));
      }
      for (int j = 0; ok && j < nk_max; ++j) {
        const int vs = j % VST;
        ok = __all_sync(FULL, mbar_wait_inl(bar(B_VFULL + vs), (j / VST) & 1, ab, kDevErrTimeout));
        if (!ok) break;
        tc_fence_after();
        if (j < nk0) {
          ok = __all_sync(FULL, mbar_wait_inl(bar(B_PFULL + 0), j & 1, ab, kDevErrTimeout));
          if (!ok) break;
          tc_fence_after();
          issue_PV(0, j);
          if (j + 1 == nk0) tc_commit_elect(bar(B_OFINAL + 0));
        }
        // S_1(j+1) overwrites the columns P_0(j) occupies (O_0 += P_0(j) V_j was
        // issued first; tcgen05.mma ops of one thread run in order) and needs
        // tile 1 to have read S_1(j)
        if (j + 1 < nk1) {
          if (!(ok = kwait(j + 1) && wait_loaded(1, j))) break;
          issue_S(1, j + 1);
          tc_commit_elect(bar(B_KEMPTY + (j + 1) % KST));
        }
        if (j < nk1) {
          ok = __all_sync(FULL, mbar_wait_inl(bar(B_PFULL + 1), j & 1, ab, kDevErrTimeout));
          if (!ok) break;
          tc_fence_after();
          issue_PV(1, j);
          if (j + 1 == nk1) tc_commit_elect(bar(B_OFINAL + 1));
        }
        // S_0(j+2): after O_1 += P_1(j) V_j (P_1(j) sits in S_0's columns) and
        // tile 0's read of S_0(j+1)
        if (j + 2 < nk0) {
          if (!(ok = kwait(j + 2) && wait_loaded(0, j + 1))) break;
          issue_S(0, j + 2);
          if (j + 2 >= nk1) tc_commit_elect(bar(B_KEMPTY + (j + 2) % KST));
        }
        tc_commit_elect(bar(B_VEMPTY + vs));
      }
      // Every MMA issued by this CTA completes before TMEM is released.
      tc_commit_elect(bar(B_FINAL));
      __syncwarp();
      drain_wait(bar(B_FINAL), 0);
      __syncwarp();
    }
  } else {
    reg_alloc<REG_SOFTMAX>();
    if (start_ok) {
        // ---------------------------------------------------------------- softmax
        const int t = warp >> 2;
        const int wq = warp & 3;
        const int r = wq * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
        const uint32_t tS = tmem + static_cast<uint32_t>(t * 128) + lane_off;
        const uint32_t tP = tmem + static_cast<uint32_t>((1 - t) * 128 + 64) + lane_off;
        const uint32_t tO = tmem + 256u + static_cast<uint32_t>(t * 128) + lane_off;
        const int my_row0 = t ? row0[1] : row0[0];
        const int my_nk = t ? nk[1] : nk[0];
        const int j_mask = first_masked_tile(a, my_row0);
        const int qrow = my_row0 + r;
        const long long qpos = a.q_offset + qrow;
        const float sl2 = a.scale_log2;
        if (a.qrot) {
          // RoPE at load: this thread's query row, rotated in fp32 at its position,
          // rounded to bf16, into the sorted-pair Q slabs (level i = HF pairs
          // 8(7-i)..8(7-i)+7); rows past the end are zero
          uint8_t* qt = sp + OFF_Q + t * QTILE_BYTES + r * 16;
          const bool valid = my_nk > 0 && qrow < row_end;
          const __nv_bfloat16* xr = a.q + static_cast<long long>(bi) * a.q_sb + static_cast<long long>(qrow) * a.q_ss +
                                    static_cast<long long>(h) * a.q_sh;
          const float* cr = a.qcos + qpos * a.cs_stride;
          const float* sr = a.qsin + qpos * a.cs_stride;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (valid) ropemath::rotate_chunk_sorted_words(xr, cr, sr, c, w);
            uint8_t* slab = qt + (7 - c) * QSLAB_BYTES;
            *reinterpret_cast<uint4*>(slab) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4*>(slab + QHALF_BYTES) = make_uint4(w[4], w[5], w[6], w[7]);
          }
          // the MMAs read Q through the async proxy
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          mbar_arrive(bar(B_Q));
        }
        float m2 = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < my_nk; ++j) {
          ok = __all_sync(FULL, mbar_wait_inl(bar(B_SFULL + t), j & 1, ab, kDevErrTimeout));
          if (!ok) break;
          tc_fence_after();
          float s[BN];
          {
            uint32_t rr[BN];
            tmem_ld128(tS, rr);
#pragma unroll
            for (int e = 0; e < BN; ++e) s[e] = __uint_as_float(rr[e]);
          }
          // S_t's columns are free now: the MMA warp may compute S_t(j+1) into
          // them, and the other tile may store its P there
          tc_fence_before();
          mbar_arrive(bar(B_LOADED + t));
          if (j >= j_mask) {
            const long long n0 = static_cast<long long>(j) * BN;
#pragma unroll
            for (int c = 0; c < BN; ++c) {
              const long long key = n0 + c;
              if ((a.causal && key > qpos) || key >= a.Sk) s[c] = -INFINITY;
            }
          }
          // three-input max: 64 instructions for the 128 scores, 4 chains
          float mx0 = fmax3(s[0], s[1], s[2]), mx1 = fmax3(s[3], s[4], s[5]);
          float mx2 = fmax3(s[6], s[7], s[8]), mx3 = fmax3(s[9], s[10], s[11]);
#pragma unroll
          for (int c = 12; c < BN - 8; c += 8) {
            mx0 = fmax3(mx0, s[c], s[c + 1]);
            mx1 = fmax3(mx1, s[c + 2], s[c + 3]);
            mx2 = fmax3(mx2, s[c + 4], s[c + 5]);
            mx3 = fmax3(mx3, s[c + 6], s[c + 7]);
          }
          mx0 = fmax3(mx0, s[BN - 4], s[BN - 3]);
          mx1 = fmax3(mx1, s[BN - 2], s[BN - 1]);
          const float mnew = fmaxf(m2, fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2);
          // Lazy rescale: the running max only moves when it grows by more than
          // 8 (log2 units), so P <= 2^8 stays exact enough in bf16 and O is
          // rescaled rarely. The O update itself happens after P is stored.
          float alpha = 1.0f;
          bool need = false;
          if (j == 0) {
            m2 = mnew;
          } else {
            need = mnew > m2 + 8.0f;
            if (need) {
              alpha = ex2_approx(m2 - mnew);
              l *= alpha;
              m2 = mnew;
            }
          }
          const float msub = (m2 == -INFINITY) ? 0.f : m2;
          // exponentials, the row sum and the bf16 packing of P, two columns at a
          // time with packed f32x2 arithmetic (half the FMA / add instructions)
          uint32_t pk[BN / 2];
          float2 ls0 = make_float2(0.f, 0.f), ls1 = make_float2(0.f, 0.f);
          const float2 sl2x2 = make_float2(sl2, sl2), negm = make_float2(-msub, -msub);
#pragma unroll
          for (int c = 0; c < BN / 2; ++c) {
            const float2 x = __ffma2_rn(make_float2(s[2 * c], s[2 * c + 1]), sl2x2, negm);
            const float2 p = make_float2(ex2_approx(x.x), ex2_approx(x.y));
            if (c & 1) ls1 = __fadd2_rn(ls1, p); else ls0 = __fadd2_rn(ls0, p);
            pk[c] = pack_bf16x2(p.x, p.y);
          }
          {
            const float2 ls = __fadd2_rn(ls0, ls1);
            l += ls.x + ls.y;
          }
          // P_t(j) goes into columns 64..127 of the other tile's S once the scores
          // there have been read: S_1(j) for tile 0, S_0(j+1) for tile 1 (whose
          // computation followed O_1 += P_1(j-1) V, the last reader of those
          // columns). Past the other tile's last key tile, wait for its last read
          // and for this tile's previous O += P V instead.
          {
            const int other_nk = t ? nk[0] : nk[1];
            const int want = j + t;  // tile 0: S_1(j); tile 1: S_0(j + 1)
            bool w = true;
            if (want < other_nk) {
              w = mbar_wait_inl(bar(B_LOADED + (t ^ 1)), want & 1, ab, kDevErrTimeout);
            } else {
              if (other_nk > 0) w = mbar_wait_inl(bar(B_LOADED + (t ^ 1)), (other_nk - 1) & 1, ab, kDevErrTimeout);
              if (w && j > 0) w = mbar_wait_inl(bar(B_ODONE + t), (j - 1) & 1, ab, kDevErrTimeout);
            }
            ok = __all_sync(FULL, w);
            if (!ok) break;
            tc_fence_after();
          }
          tmem_st64(tP, pk);
          if (__any_sync(FULL, need)) {
            // O holds the sum up to tile j-1 once PV(t, j-1) has completed (S_t(j) was
            // issued after it, so at most that one is in flight); PV(t, j) is not
            // issued before this warpgroup arrives on PFULL below.
            ok = __all_sync(FULL, mbar_wait_inl(bar(B_ODONE + t), (j - 1) & 1, ab, kDevErrTimeout));
            if (!ok) break;
            tc_fence_after();
#pragma unroll
            for (int c4 = 0; c4 < HD / 32; ++c4) {
              uint32_t rr[32];
              tmem_ld32(tO + static_cast<uint32_t>(32 * c4), rr);
#pragma unroll
              for (int e = 0; e < 32; ++e) rr[e] = __float_as_uint(__uint_as_float(rr[e]) * alpha);
              tmem_st32(tO + static_cast<uint32_t>(32 * c4), rr);
            }
          }
          tc_fence_before();
          mbar_arrive(bar(B_PFULL + t));
        }
        if (ok && my_nk > 0) {
          ok = __all_sync(FULL, mbar_wait_inl(bar(B_OFINAL + t), 0, ab, kDevErrTimeout));
          if (ok) {
            tc_fence_after();
            const float inv = l > 0.f ? 1.0f / l : 0.f;
            const bool store = qrow < row_end;
            __nv_bfloat16* orow = a.out + static_cast<long long>(bi) * a.o_sb +
                                  static_cast<long long>(qrow) * a.o_ss +
                                  static_cast<long long>(h) * a.o_sh;
#pragma unroll
            for (int c4 = 0; c4 < HD / 32; ++c4) {
              uint32_t rr[32];
              tmem_ld32(tO + static_cast<uint32_t>(32 * c4), rr);
              uint32_t pk[16];
#pragma unroll
              for (int e = 0; e < 16; ++e)
                pk[e] = pack_bf16x2(__uint_as_float(rr[2 * e]) * inv, __uint_as_float(rr[2 * e + 1]) * inv);
              if (store) {
                uint4* dst = reinterpret_cast<uint4*>(orow + 32 * c4);
#pragma unroll
                for (int v4 = 0; v4 < 4; ++v4)
                  dst[v4] = make_uint4(pk[4 * v4], pk[4 * v4 + 1], pk[4 * v4 + 2], pk[4 * v4 + 3]);
              }
            }
            if (a.lse != nullptr && store)
              a.lse[(static_cast<long long>(bi) * a.Hq + h) * a.Sq + qrow] =
                  (m2 + log2f(l)) * 0.69314718055994531f;
          }
        }
    }
  }

  __syncthreads();
  if (warp == WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace prefill
}  // namespace atf

using namespace atf;

extern "C" int atf_prefill_fwd(const AtfPrefillParams* p, atf_stream_t stream) {
  using namespace atf::prefill;
  if (p == nullptr || p->q == nullptr || p->k == nullptr || p->v == nullptr || p->out == nullptr)
    return ATF_ERR_INVALID_ARG;
  if (p->head_dim != ATF_HEAD_DIM) return ATF_ERR_UNSUPPORTED;
  if (p->batch < 1 || p->seqlen_q < 1 || p->seqlen_k < 1 || p->num_heads_q < 1 ||
      p->num_heads_kv < 1 || p->num_heads_q % p->num_heads_kv != 0)
    return ATF_ERR_INVALID_ARG;
  if (p->seqlen_q > (1ll << 30) || p->seqlen_k > (1ll << 30) || p->batch * p->num_heads_q > (1 << 20))
    return ATF_ERR_UNSUPPORTED;
  if (p->causal && p->q_offset < 0) return ATF_ERR_UNSUPPORTED;
  if (p->q_offset < 0 || p->q_offset + p->seqlen_q > (1ll << 31)) return ATF_ERR_INVALID_ARG;
  if (p->qk_layout != ATF_LAYOUT_SORTED_PAIR && p->qk_layout != ATF_LAYOUT_ROTATE_HALF)
    return ATF_ERR_INVALID_ARG;
  if (p->window != ATF_WINDOW_OFF && p->window != ATF_WINDOW_SNAP16) return ATF_ERR_UNSUPPORTED;
  if (!(p->softmax_scale > 0.f)) return ATF_ERR_INVALID_ARG;
  if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->out))
    return ATF_ERR_ALIGNMENT;
  const int64_t strides[12] = {p->q_stride_b, p->q_stride_s, p->q_stride_h, p->k_stride_b,
                               p->k_stride_s, p->k_stride_h, p->v_stride_b, p->v_stride_s,
                               p->v_stride_h, p->o_stride_b, p->o_stride_s, p->o_stride_h};
  for (int i = 0; i < 12; ++i)
    if (strides[i] < 0 || (strides[i] & 7) != 0) return ATF_ERR_ALIGNMENT;
  const bool qrot = p->q_cos != nullptr || p->q_sin != nullptr;
  if (qrot) {
    // q is pre-RoPE rotate_half; k must already be post-RoPE sorted pairs
    if (p->q_cos == nullptr || p->q_sin == nullptr || p->qk_layout != ATF_LAYOUT_SORTED_PAIR ||
        p->q_cs_stride_pos < 64 || p->q_n_pos < p->q_offset + p->seqlen_q)
      return ATF_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(p->q_cos) & 3) || (reinterpret_cast<uintptr_t>(p->q_sin) & 3))
      return ATF_ERR_ALIGNMENT;
  }
  if (p->window == ATF_WINDOW_SNAP16) {
    for (int i = 0; i < ATF_MAX_LEVELS; ++i)
      if (p->zhi[i] < 0 || (i > 0 && p->zhi[i] > p->zhi[i - 1])) return ATF_ERR_INVALID_ARG;
    // zhi[0] must cover the largest distance in the problem (D_eff >= 16 always).
    if (static_cast<int64_t>(p->zhi[0]) < p->q_offset + p->seqlen_q - 1) return ATF_ERR_INVALID_ARG;
  }
  if (p->num_row_ranges < 0 || p->num_row_ranges > 2) return ATF_ERR_INVALID_ARG;
  for (int r = 0; r < p->num_row_ranges; ++r) {
    const int64_t lo = p->row_begin[r], hi = p->row_end[r];
    if (lo < 0 || hi <= lo || hi > p->seqlen_q || (lo % BM) != 0) return ATF_ERR_INVALID_ARG;
    if (r > 0 && lo < p->row_end[r - 1]) return ATF_ERR_INVALID_ARG;
  }
  int dev = 0;
  int rc = check_device(&dev);
  if (rc != ATF_OK) return rc;

  CUtensorMap tq, tk, tv;
  KLevelMaps tkl;
  auto sane = [](int64_t stride, int64_t size) -> uint64_t {
    // Size-1 dims may carry any stride; use a valid placeholder.
    return static_cast<uint64_t>(size == 1 ? 16 : stride * 2);
  };
  {
    const uint64_t dims[4] = {128, (uint64_t)p->seqlen_q, (uint64_t)p->num_heads_q, (uint64_t)p->batch};
    const uint64_t str[3] = {sane(p->q_stride_s, p->seqlen_q), sane(p->q_stride_h, p->num_heads_q),
                             sane(p->q_stride_b, p->batch)};
    const uint32_t box[4] = {8, static_cast<uint32_t>(BM), 1, 1};
    if ((rc = encode_tiled_bf16(&tq, p->q, 4, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE)) != ATF_OK)
      return rc;
  }
  {
    const uint64_t dims[4] = {128, (uint64_t)p->seqlen_k, (uint64_t)p->num_heads_kv, (uint64_t)p->batch};
    const uint64_t str[3] = {sane(p->k_stride_s, p->seqlen_k), sane(p->k_stride_h, p->num_heads_kv),
                             sane(p->k_stride_b, p->batch)};
    const uint32_t box[4] = {8, static_cast<uint32_t>(BN), 1, 1};
    if ((rc = encode_tiled_bf16(&tk, p->k, 4, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE)) != ATF_OK)
      return rc;
    // (16 dims, key, level, kv head, batch): the level axis is a view of head_dim
    const uint64_t dims5[5] = {16, (uint64_t)p->seqlen_k, ATF_MAX_LEVELS, (uint64_t)p->num_heads_kv,
                               (uint64_t)p->batch};
    const uint64_t str5[4] = {sane(p->k_stride_s, p->seqlen_k), 32, sane(p->k_stride_h, p->num_heads_kv),
                              sane(p->k_stride_b, p->batch)};
    for (int L = 1; L <= ATF_MAX_LEVELS; ++L) {
      const uint32_t box5[5] = {16, static_cast<uint32_t>(BN), static_cast<uint32_t>(L), 1, 1};
      if ((rc = encode_tiled_bf16(&tkl.lv[L - 1], p->k, 5, dims5, str5, box5, CU_TENSOR_MAP_SWIZZLE_32B)) != ATF_OK)
        return rc;
    }
  }
  {
    const uint64_t dims[4] = {128, (uint64_t)p->seqlen_k, (uint64_t)p->num_heads_kv, (uint64_t)p->batch};
    const uint64_t str[3] = {sane(p->v_stride_s, p->seqlen_k), sane(p->v_stride_h, p->num_heads_kv),
                             sane(p->v_stride_b, p->batch)};
    const uint32_t box[4] = {64, static_cast<uint32_t>(BN), 1, 1};
    if ((rc = encode_tiled_bf16(&tv, p->v, 4, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) != ATF_OK)
      return rc;
  }

  Args a;
  a.B = static_cast<int>(p->batch);
  a.Sq = static_cast<int>(p->seqlen_q);
  a.Sk = static_cast<int>(p->seqlen_k);
  a.Hq = static_cast<int>(p->num_heads_q);
  a.G = static_cast<int>(p->num_heads_q / p->num_heads_kv);
  if (p->num_row_ranges == 0) {
    a.nrange = 1;
    a.r_lo[0] = 0;
    a.r_hi[0] = static_cast<int>(p->seqlen_q);
  } else {
    a.nrange = p->num_row_ranges;
    for (int r = 0; r < a.nrange; ++r) {
      a.r_lo[r] = static_cast<int>(p->row_begin[r]);
      a.r_hi[r] = static_cast<int>(p->row_end[r]);
    }
  }
  a.n_qblk = 0;
  for (int r = 0; r < 2; ++r) {
    a.r_nblk[r] = r < a.nrange ? (a.r_hi[r] - a.r_lo[r] + BM * NQ - 1) / (BM * NQ) : 0;
    if (r >= a.nrange) a.r_lo[r] = a.r_hi[r] = 0;
    a.n_qblk += a.r_nblk[r];
  }
  a.q_offset = p->q_offset;
  a.scale_log2 = p->softmax_scale * 1.4426950408889634f;
  a.causal = p->causal ? 1 : 0;
  a.layout = p->qk_layout;
  a.window = p->window == ATF_WINDOW_SNAP16 ? 1 : 0;
  for (int i = 0; i < ATF_MAX_LEVELS; ++i) a.zhi[i] = p->zhi[i];
  a.out = static_cast<__nv_bfloat16*>(p->out);
  a.o_sb = p->o_stride_b;
  a.o_ss = p->o_stride_s;
  a.o_sh = p->o_stride_h;
  a.lse = p->lse;
  a.err = p->error_flag;
  a.qrot = qrot ? 1 : 0;
  a.q = static_cast<const __nv_bfloat16*>(p->q);
  a.q_sb = p->q_stride_b;
  a.q_ss = p->q_stride_s;
  a.q_sh = p->q_stride_h;
  a.qcos = p->q_cos;
  a.qsin = p->q_sin;
  a.cs_stride = p->q_cs_stride_pos;

  if (cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(SMEM_BYTES)) != cudaSuccess)
    return ATF_ERR_CUDA;
  const long long grid = static_cast<long long>(a.n_qblk) * a.B * a.Hq;
  if (grid > 0x7fffffffLL) return ATF_ERR_UNSUPPORTED;
  // setmaxnreg.inc waits until the block's launch registers cover the split:
  // never launch a build whose register count would leave it waiting
  static const int launch_regs = [] {
    cudaFuncAttributes fa{};
    return cudaFuncGetAttributes(&fa, prefill_kernel) == cudaSuccess ? fa.numRegs : 0;
  }();
  if (static_cast<long long>(launch_regs) * THREADS < REG_SPLIT_TOTAL) return ATF_ERR_UNSUPPORTED;
  prefill_kernel<<<static_cast<unsigned>(grid), THREADS, SMEM_BYTES,
                   reinterpret_cast<cudaStream_t>(stream)>>>(tq, tk, tkl, tv, a);
  return cudaGetLastError() == cudaSuccess ? ATF_OK : ATF_ERR_CUDA;
}
