// Persistent, warp-specialised causal prefill on tcgen05 + TMEM.
//
// Same mathematics, operand layouts and MMA descriptors as prefill_tc2_kernel
// (two 128-row query tiles A and B of one (head, sequence) share every K/V
// tile; S = Q K^T and O += P V on the tensor cores with fp32 accumulators in
// tensor memory; P written back over S as bf16/fp16 and read by the P.V MMA
// straight from tensor memory; the running max raised lazily), scheduled
// differently:
//
//   * Persistent grid: one CTA per SM walks work units (256 query rows, query
//     head, sequence) in a static order that puts the units with the most KV
//     tiles first (the last query blocks of the longest sequences), so the
//     causal triangle's long units start early and short ones fill the tail.
//     Tensor memory is allocated once per CTA, not once per unit.
//   * Sixteen warps in four warpgroups: warps 0-3 and 4-7 run the softmax of
//     tiles A and B (thread = query row = TMEM lane; warp w reaches lanes
//     32 (w mod 4) .. +31), warps 8-11 write out O (the epilogue), warp 12
//     issues TMA loads and warp 13 the MMAs (each runs its loop warp-wide,
//     so the operands stay warp-uniform, and one elected lane issues),
//     warps 14-15 only take part in the register split.  `setmaxnreg` moves registers from the
//     epilogue and issuing warpgroups to the softmax warpgroups, which hold a
//     row's 128 scores in registers.  K and V have separate two-stage rings
//     with their own "free" barriers: K_j is released as soon as both S MMAs
//     that read it finish, V_j after both P.V MMAs.
//   * A softmax thread loads its 128 scores from tensor memory with four
//     loads and one wait, keeps them in registers for the max and the
//     exponentials, and stores P back with four stores and one wait.
//   * The next unit's Q tiles load as soon as the current unit's last S MMA
//     has finished; its first S MMAs and softmax run while the epilogue
//     warps read out the current unit's O (the row sums reach them through
//     shared memory, double-buffered by unit; tensor memory O is handed back
//     to the MMA warp through an "O free" barrier once read).
//
// Every wait is bounded (kWaitLimitNs).  A role that gives up sets an abort
// flag in shared memory and records NB_DEVERR_TIMEOUT; every role checks the
// flag between steps and leaves the unit loop; before the CTA exits the
// producer waits (bounded) for its copies in flight and the MMA warp for its
// MMAs, then tensor memory is freed.
#pragma once
#include <climits>
#include <type_traits>

#include "nb_common.cuh"

namespace nb {

// 2^x for two values on the FMA/ALU pipes (packed fp32 pairs), for a share
// of the softmax exponentials that would otherwise queue on the MUFU (XU)
// pipe.  Cody-Waite style range reduction: n = round(x) through the
// 1.5 * 2^23 magic constant, f = x - n in [-0.5, 0.5] (formed as n * -1 + x,
// one rounding as a subtraction); 2^f by a cubic whose coefficients were fit
// here (least squares weighted by relative error on [-0.5, 0.5], maximum
// relative error 1.0e-4, below half a unit of bf16 and fp16); 2^n is added
// to the exponent field.  Valid for x >= -126 (the unmasked scores, which
// are at most a few units above the running max).
__device__ __forceinline__ void exp2_poly2(float& y0, float& y1, float x0, float x1) {
  x0 = fmaxf(x0, -126.f);
  x1 = fmaxf(x1, -126.f);
  float t0, t1, n0, n1, f0, f1, p0, p1;
  add_f32x2(t0, t1, x0, x1, 12582912.f, 12582912.f);
  add_f32x2(n0, n1, t0, t1, -12582912.f, -12582912.f);
  fma_f32x2(f0, f1, n0, n1, -1.f, -1.f, x0, x1);
  fma_f32x2(p0, p1, f0, f1, 0.05500858144334074f, 0.05500858144334074f, 0.24221037434204812f,
            0.24221037434204812f);
  fma_f32x2(p0, p1, p0, p1, f0, f1, 0.6932829004942702f, 0.6932829004942702f);
  fma_f32x2(p0, p1, p0, p1, f0, f1, 1.0f, 1.0f);
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

// Value pairs (of every 8) that take exp2_poly2 instead of the MUFU in a
// warp whose rows are all unmasked; 0 by default (measured slower: the
// softmax warps spill at 168 registers with both paths in the loop).
#ifndef NB_PF3_POLY
#define NB_PF3_POLY 0
#endif

template <int D> struct Pf3Geom {
  static constexpr int kAtom = 128 * 128;       // 128 rows x 128 B
  static constexpr int kTile = (D / 64) * kAtom;
  static constexpr int kQA = 0;
  static constexpr int kQB = kTile;
  static constexpr int kK = 2 * kTile;          // K ring: 2 stages
  static constexpr int kV = kK + 2 * kTile;     // V ring: 2 stages
  static constexpr int kBars = kV + 2 * kTile;
  // row sums handed from the softmax groups to the epilogue:
  // [group][unit parity][row] floats
  static constexpr int kRowSum = kBars + 256;
  // the epilogue's staging box for a TMA store of O: 128 rows x 64 columns,
  // 128-byte swizzle (1024-byte aligned)
  static constexpr int kOStage = kRowSum + 3072 - 256;
  static constexpr int kSmem = kOStage + kAtom + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kSA = 0, kSB = 128, kOA = 256, kOB = 256 + D;
};
// Warp roles (four warpgroups; a warp reaches the TMEM lanes 32 (w mod 4) ..
// +31) and the register split between them.  The block is launched with
// kPf3Threads x kPf3LaunchRegs registers (the whole register file); the
// shares after `setmaxnreg` add up to exactly that (checked below and, on
// the host, against the compiled kernel before the first launch).
constexpr int kPf3Threads = 512;
constexpr int kPf3LaunchRegs = 128;
constexpr int kPf3SoftmaxRegs = 168;   // warpgroups 0, 1
constexpr int kPf3EpilogueRegs = 72;   // warpgroup 2
constexpr int kPf3IssueRegs = 104;     // warpgroup 3 (TMA, MMA, two idle warps)
static_assert(128 * (2 * kPf3SoftmaxRegs + kPf3EpilogueRegs + kPf3IssueRegs) <=
                  kPf3Threads * kPf3LaunchRegs,
              "the register split must fit the registers the block is launched with");
static_assert(kPf3Threads * kPf3LaunchRegs <= 65536, "one CTA per SM");
constexpr int kPf3WarpEpi = 8, kPf3WarpTma = 12, kPf3WarpMma = 13;

template <int N> __device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N> __device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// max(a, b, c) in one instruction (sm_100 three-input max; NaN handling as
// fmaxf: a NaN operand is ignored).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Paged mode: K and V come from the paged cache [2, N, kvh, 16, D] through
// the block table (keys 0 .. ctx + len - 1 of a sequence: the cached prefix
// and the new tokens, whose rows the KV writer stored first), and query row i
// of a sequence sits at absolute position ctx + i.  bt == nullptr: K and V
// are the new tokens' contiguous rows and ctx = 0 (needle's prefill).
struct Pf3Paged {
  const int32_t* bt;    // [B, bt_stride] block ids
  int64_t bt_stride;
  int maxb;             // block-table columns
  const int32_t* ctx;   // [B] cached tokens before the new ones
  int num_blocks, kvh;
};

// Work unit u -> (query block, head, sequence); units with the most KV tiles
// come first.  Units past a sequence's end are empty (every role skips them).
// Two ways to give the two softmax groups their 128-row query tiles:
//   pair = 0: the two halves of a 256-row block of one head (tile B sees one
//             KV tile more than tile A);
//   pair = 1: one 128-row block of two heads that share a KV head (even GQA
//             groups): both tiles see the same KV tiles, so the groups stay
//             in step to the unit's end and every K/V tile serves both.
struct Pf3Unit {
  int qb, h, b;  // h: the head of tile A (pair = 1: tile B is head h + 1)
};
__device__ __forceinline__ Pf3Unit pf3_unit(int u, int hq, int B, int nqb, int pair) {
  const int hu = pair ? hq / 2 : hq;
  const int per = hu * B;
  const int r = u % per;
  return Pf3Unit{nqb - 1 - u / per, (r % hu) * (pair ? 2 : 1), r / hu};
}
// First query row (within the sequence) and head of tile x of a unit.
__device__ __forceinline__ int pf3_row(const Pf3Unit& w, int x, int pair) {
  return pair ? w.qb * 128 : w.qb * 256 + x * 128;
}
__device__ __forceinline__ int pf3_head(const Pf3Unit& w, int x, int pair) {
  return pair ? w.h + x : w.h;
}

template <typename T, int D>
__global__ void __launch_bounds__(kPf3Threads, 1)
    prefill_tc3_kernel(const __grid_constant__ CUtensorMap qmap,
                       const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap, const int32_t* __restrict__ cu,
                       int B, int hq, int group, int nqb, int pair, float scale_log2,
                       T* __restrict__ out, int64_t os, const Pf3Paged pg,
                       const __grid_constant__ CUtensorMap omap, int o_tma) {
  using G = Pf3Geom<D>;
  static_assert(G::kOStage % 1024 == 0 && G::kOStage >= G::kRowSum + 2 * 2 * 128 * 4,
                "staging box placement");
  constexpr bool kBf16 = !__is_same(T, __half);
  constexpr uint32_t kIdS = idesc_f16_f32(kBf16, 128, 128, false, false);
  constexpr uint32_t kIdO = idesc_f16_f32(kBf16, 128, D, false, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sb = smem_u32(smem);
  // barriers (8 bytes each)
  const uint32_t bar_q = sb + G::kBars;            // Q_A (+Q_B) landed
  const uint32_t bar_k = bar_q + 8;                // [2] K stage landed
  const uint32_t bar_v = bar_q + 24;               // [2] V stage landed
  const uint32_t bar_kfree = bar_q + 40;           // [2] K stage read by its S MMAs
  const uint32_t bar_vfree = bar_q + 56;           // [2] V stage read by its P.V MMAs
  const uint32_t bar_qfree = bar_q + 72;           // this unit's S MMAs done: Q may reload
  const uint32_t bar_s = bar_q + 80;               // [2] S_A / S_B ready
  const uint32_t bar_p = bar_q + 96;               // [2] P_A / P_B written (128 arrivals)
  const uint32_t bar_o = bar_q + 112;              // [2] O_A / O_B final
  const uint32_t bar_ofree = bar_q + 128;          // [2] O_A / O_B read out (128 arrivals)
  const uint32_t bar_end = bar_q + 144;            // every MMA of the CTA finished
  const uint32_t bar_l = bar_q + 152;              // [group][unit parity] row sums written
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + G::kBars + 192);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::kBars + 200);
  float* rowsum = reinterpret_cast<float*>(smem + G::kRowSum);  // [2][2][128]

  if (warp == kPf3WarpMma) {
    tmem_alloc(smem_u32(tmem_slot), G::kTmemCols);
    tmem_relinquish();
  }
  if (warp == kPf3WarpTma && lane == 0) {
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    mbar_init(bar_q, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_k + 8 * i, 1);
      mbar_init(bar_v + 8 * i, 1);
      mbar_init(bar_kfree + 8 * i, 1);
      mbar_init(bar_vfree + 8 * i, 1);
      mbar_init(bar_s + 8 * i, 1);
      mbar_init(bar_p + 8 * i, 128);
      mbar_init(bar_o + 8 * i, 1);
      mbar_init(bar_ofree + 8 * i, 128);
    }
    for (int i = 0; i < 4; ++i) mbar_init(bar_l + 8 * i, 128);
    mbar_init(bar_qfree, 1);
    mbar_init(bar_end, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_units = nqb * (pair ? hq / 2 : hq) * B;

  // This CTA's units: round rd takes unit rd * G + blockIdx.x, or, in odd
  // rounds, rd * G + G - 1 - blockIdx.x (the units are sorted by size, so
  // alternating the direction evens out the CTAs' totals: 3 % shorter than
  // plain round-robin on the worst CTA at 16 x 1024).
  auto unit_of = [&](int rd) -> int {
    return rd * (int)gridDim.x +
           ((rd & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x);
  };
  const bool paged = pg.bt != nullptr;
  // keys a sequence can have: the block table's pages (as decode, which reads
  // at most max_blocks pages of a longer context)
  const int kcap = paged ? pg.maxb * 16 : INT_MAX;
  // Causal extent of a unit: KV tiles under tile A / tile B (0: no tile B);
  // c = the sequence's cached prefix (keys before its new tokens)
  auto extent = [&](const Pf3Unit& w, int& s0, int& len, int& nA, int& nB, int& c) -> bool {
    s0 = __ldg(cu + w.b);
    len = __ldg(cu + w.b + 1) - s0;
    c = paged ? max(0, __ldg(pg.ctx + w.b)) : 0;
    const int q0 = pf3_row(w, 0, pair);
    if (q0 >= len) return false;
    const int q1 = pf3_row(w, 1, pair);
    const int klast = min(c + len, kcap) - 1;  // last key of the sequence
    nA = (min(c + q0 + 127, klast) >> 7) + 1;
    nB = q1 < len ? (min(c + q1 + 127, klast) >> 7) + 1 : 0;
    return true;
  };
  // paged mode: first cache row (K half) of page p of sequence b for KV head
  // kh, or -16 (a box wholly before the tensor: TMA fills zeros) for a page
  // past the table or an invalid block id (recorded)
  auto page_row = [&](int b, int p, int kh) -> int {
    if (p >= pg.maxb) return -16;
    const int phys = __ldg(pg.bt + (int64_t)b * pg.bt_stride + p);
    if (phys < 0 || phys >= pg.num_blocks) {
      set_error(kErrBlockId);
      return -16;
    }
    return (phys * pg.kvh + kh) * 16;
  };

  const int wg = warp >> 2;
  if (wg == 3) {
    setmaxnreg_dec<kPf3IssueRegs>();
  if (warp == kPf3WarpTma) {
    // ---------------- TMA producer: the whole warp runs the loop, one
    // elected lane issues the copies ----------------
    {
      uint32_t nq = 0, nk = 0, nv = 0;  // loads issued (running counts)
      bool ok = true;
      // one answer for the warp, which takes every branch together
      auto wait = [&](uint32_t bar, uint32_t par) {
        return __all_sync(0xffffffffu, mbar_wait_bounded(bar, par));
      };
      for (int rd = 0, u = unit_of(0); ok && u < n_units; u = unit_of(++rd)) {
        const Pf3Unit w = pf3_unit(u, hq, B, nqb, pair);
        int s0, len, nA, nB, c;
        if (!extent(w, s0, len, nA, nB, c)) continue;
        const int kh = w.h / group;
        const int n_kv = nB ? nB : nA;
        if (nq > 0 && !wait(bar_qfree, (nq - 1) & 1)) { ok = false; break; }
        if (elect_one()) {
          mbar_arrive_expect_tx(bar_q, (nB ? 2 : 1) * G::kTile);
#pragma unroll
          for (int a = 0; a < D / 64; ++a) {
            tma_load_2d(sb + G::kQA + a * G::kAtom, &qmap, pf3_head(w, 0, pair) * D + a * 64,
                        s0 + pf3_row(w, 0, pair), bar_q);
            if (nB)
              tma_load_2d(sb + G::kQB + a * G::kAtom, &qmap, pf3_head(w, 1, pair) * D + a * 64,
                          s0 + pf3_row(w, 1, pair), bar_q);
          }
        }
        ++nq;
        for (int j = 0; j < n_kv; ++j) {
          if (__any_sync(0xffffffffu, *abort_flag)) { ok = false; break; }
          const uint32_t st = nk & 1;
          if (nk >= 2 && !wait(bar_kfree + 8 * st, ((nk >> 1) - 1) & 1)) {
            ok = false;
            break;
          }
          // paged: the tile's 8 pages (16 keys each) through the block table;
          // a 16-row box at a 16-row offset keeps the 128-byte swizzle of the
          // 128-row tile
          int prow[8];
          if (paged) {
#pragma unroll
            for (int pp = 0; pp < 8; ++pp) prow[pp] = page_row(w.b, j * 8 + pp, kh);
          }
          const int v_off = paged ? pg.num_blocks * pg.kvh * 16 : 0;
          if (elect_one()) {
            mbar_arrive_expect_tx(bar_k + 8 * st, G::kTile);
#pragma unroll
            for (int a = 0; a < D / 64; ++a) {
              const uint32_t dst = sb + G::kK + st * G::kTile + a * G::kAtom;
              if (paged) {
#pragma unroll
                for (int pp = 0; pp < 8; ++pp)
                  tma_load_2d(dst + pp * 16 * 128, &kmap, a * 64, prow[pp], bar_k + 8 * st);
              } else {
                tma_load_2d(dst, &kmap, kh * D + a * 64, s0 + j * 128, bar_k + 8 * st);
              }
            }
          }
          ++nk;
          if (nv >= 2 && !wait(bar_vfree + 8 * st, ((nv >> 1) - 1) & 1)) {
            ok = false;
            break;
          }
          if (elect_one()) {
            mbar_arrive_expect_tx(bar_v + 8 * st, G::kTile);
#pragma unroll
            for (int a = 0; a < D / 64; ++a) {
              const uint32_t dst = sb + G::kV + st * G::kTile + a * G::kAtom;
              if (paged) {
#pragma unroll
                for (int pp = 0; pp < 8; ++pp)
                  tma_load_2d(dst + pp * 16 * 128, &kmap, a * 64,
                              prow[pp] < 0 ? prow[pp] : prow[pp] + v_off, bar_v + 8 * st);
              } else {
                tma_load_2d(dst, &vmap, kh * D + a * 64, s0 + j * 128, bar_v + 8 * st);
              }
            }
          }
          ++nv;
        }
      }
      if (!ok && lane == 0) {
        *abort_flag = 1;
        set_error(kErrTimeout);
      }
      // copies still in flight land before the CTA may exit: wait (bounded)
      // for the last phase of every barrier a load was issued on
      if (nq) mbar_wait_bounded(bar_q, (nq - 1) & 1);
      for (uint32_t i = (nk > 2 ? nk - 2 : 0); i < nk; ++i)
        mbar_wait_bounded(bar_k + 8 * (i & 1), (i >> 1) & 1);
      for (uint32_t i = (nv > 2 ? nv - 2 : 0); i < nv; ++i)
        mbar_wait_bounded(bar_v + 8 * (i & 1), (i >> 1) & 1);
    }
  } else if (warp == kPf3WarpMma) {
    // ---------------- MMA issuer: the whole warp runs the loop, one elected
    // lane issues each MMA and commit ----------------
    {
      uint32_t nq = 0, nk = 0, nv = 0;           // tiles consumed (running counts)
      uint32_t np[2] = {0, 0}, no[2] = {0, 0};   // P tiles consumed, units finished per group
      bool ok = true;
      auto wait = [&](uint32_t bar, uint32_t par) {
        if (!ok) return false;
        // one answer for the warp, which takes every branch together
        ok = __all_sync(0xffffffffu, !*abort_flag && mbar_wait_bounded(bar, par));
        return ok;
      };
      auto commit = [&](uint32_t bar) {
        if (elect_one()) tc_commit(bar);
      };
      auto issue_s = [&](uint32_t q_off, uint32_t kst, uint32_t t_col) {
        const bool leader = elect_one();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * G::kAtom + (kk & 3) * 32;
          const uint64_t ad = smem_desc_sw128(sb + q_off + off, 16, 1024);
          const uint64_t bd = smem_desc_sw128(kst + off, 16, 1024);
          if (leader) tc_mma_f16_ss(tmem + t_col, ad, bd, kIdS, kk > 0);
        }
      };
      auto issue_pv = [&](uint32_t vst, uint32_t s_col, uint32_t o_col, bool first) {
        const bool leader = elect_one();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t bd = smem_desc_sw128(vst + kk * 16 * 128, G::kAtom, 1024);
          if (leader)
            tc_mma_f16_ts(tmem + o_col, tmem + s_col + kk * 8, bd, kIdO,
                          (!first || kk > 0) ? 1u : 0u);
        }
      };
      // the first unit at or after round rd with work (its KV tile counts)
      auto next_unit = [&](int& rd, int& tA, int& tB) -> bool {
        for (int u = unit_of(rd); u < n_units; u = unit_of(++rd)) {
          int s0, len, c;
          if (extent(pf3_unit(u, hq, B, nqb, pair), s0, len, tA, tB, c)) return true;
        }
        return false;
      };
      const uint32_t qoff[2] = {(uint32_t)G::kQA, (uint32_t)G::kQB};
      const uint32_t scol[2] = {G::kSA, G::kSB}, ocol[2] = {G::kOA, G::kOB};
      int rd = 0, nA = 0, nB = 0;
      bool have = next_unit(rd, nA, nB);
      bool first_unit = true;
      while (ok && have) {
        const int n_kv = nB ? nB : nA;
        const int nx[2] = {nA, nB};
        int rd2 = rd + 1, mA = 0, mB = 0;
        const bool have2 = next_unit(rd2, mA, mB);
        const int mx[2] = {mA, mB};
        if (first_unit) {
          // S_X(0) for both tiles (later units' are issued at the end of the
          // unit before them)
          if (!wait(bar_q, nq & 1)) break;
          ++nq;
          const uint32_t st = nk & 1;
          if (!wait(bar_k + 8 * st, (nk >> 1) & 1)) break;
          tc_fence_after();
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            if (!nx[x]) continue;
            issue_s(qoff[x], sb + G::kK + st * G::kTile, scol[x]);
            commit(bar_s + 8 * x);
          }
          commit(bar_kfree + 8 * st);
          if (n_kv == 1) commit(bar_qfree);
          ++nk;
          first_unit = false;
        }
        // the next unit's Q / K_0 landed (waited), its S_X(0) issued (bit x)
        bool q2 = false, k2 = false;
        uint32_t early = 0;
        auto next_ready = [&]() -> bool {
          if (!q2) {
            if (!wait(bar_q, nq & 1)) return false;
            q2 = true;
          }
          if (!k2) {
            if (!wait(bar_k + 8 * (nk & 1), (nk >> 1) & 1)) return false;
            tc_fence_after();
            k2 = true;
          }
          return true;
        };
        for (int j = 0; ok && j < n_kv; ++j) {
          const uint32_t vst = nv & 1;
          if (!wait(bar_v + 8 * vst, (nv >> 1) & 1)) break;
          const bool has_next = j + 1 < n_kv;
          const uint32_t kst = nk & 1;
          bool k_ready = false;
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            if (!ok) break;
            if (j >= nx[x]) continue;
            // P_X(j) written by the softmax group; O_X free on its first tile
            if (j == 0 && no[x] > 0 && !wait(bar_ofree + 8 * x, (no[x] - 1) & 1)) break;
            if (!wait(bar_p + 8 * x, np[x] & 1)) break;
            ++np[x];
            tc_fence_after();
            issue_pv(sb + G::kV + vst * G::kTile, scol[x], ocol[x], j == 0);
            if (j + 1 == nx[x]) {
              commit(bar_o + 8 * x);  // O_X final for this unit
              ++no[x];
              // At the unit's last KV tile the next unit's S_X(0) goes in
              // right behind this P.V, before the other tile's P is waited
              // for: its Q was requested when this unit's last S MMAs were
              // issued and its K_0 when the stage before it was freed, so the
              // producer needs nothing more from this warp.
              if (have2 && mx[x] && !has_next) {
                if (!next_ready()) break;
                issue_s(qoff[x], sb + G::kK + (nk & 1) * G::kTile, scol[x]);
                commit(bar_s + 8 * x);  // also covers P_X(j).V_j
                early |= 1u << x;
              }
            } else {
              if (!k_ready) {
                if (!wait(bar_k + 8 * kst, (nk >> 1) & 1)) break;
                tc_fence_after();
                k_ready = true;
              }
              issue_s(qoff[x], sb + G::kK + kst * G::kTile, scol[x]);
              commit(bar_s + 8 * x);  // also covers P_X(j).V_j
            }
          }
          if (!ok) break;
          commit(bar_vfree + 8 * vst);
          ++nv;
          if (has_next) {
            commit(bar_kfree + 8 * kst);
            if (j + 2 == n_kv) commit(bar_qfree);  // last S MMAs of the unit issued
            ++nk;
          }
        }
        if (!ok) break;
        if (have2) {
          // the next unit's remaining S_X(0) (a tile that ended before this
          // unit's last KV tile), then its Q and K_0 bookkeeping
          if (!next_ready()) break;
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            if (!mx[x] || ((early >> x) & 1u)) continue;
            issue_s(qoff[x], sb + G::kK + (nk & 1) * G::kTile, scol[x]);
            commit(bar_s + 8 * x);
          }
          ++nq;
          commit(bar_kfree + 8 * (nk & 1));
          if ((mB ? mB : mA) == 1) commit(bar_qfree);
          ++nk;
        }
        rd = rd2;
        nA = mA;
        nB = mB;
        have = have2;
      }
      if (!ok && lane == 0) {
        *abort_flag = 1;
        set_error(kErrTimeout);
      }
      commit(bar_end);
      mbar_wait_bounded(bar_end, 0);  // every MMA issued by this CTA has finished
    }
  }
  } else if (wg < 2) {
    setmaxnreg_inc<kPf3SoftmaxRegs>();
    // ---------------- softmax groups ----------------
    constexpr int NCC = 4;                 // 32-column TMEM chunks of a row's 128 scores
    constexpr int OC = D / 32;             // 32-column O chunks
    const int x = wg;                      // 0 = tile A, 1 = tile B
    // A warp reaches the TMEM lanes of its warp index mod 4: lanes [32 wq,
    // 32 wq + 32); a thread's query row is its TMEM lane.
    const int wq = warp & 3;
    const uint32_t tS = tmem + (x ? G::kSB : G::kSA);
    const uint32_t tO = tmem + (x ? G::kOB : G::kOA);
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const int r = wq * 32 + lane;
    uint32_t ns = 0, nunits = 0;
    bool ok = true;
    for (int rd = 0, u = unit_of(0); ok && u < n_units; u = unit_of(++rd)) {
      const Pf3Unit w = pf3_unit(u, hq, B, nqb, pair);
      int s0, len, nA, nB, c;
      if (!extent(w, s0, len, nA, nB, c)) continue;
      const int n_mine = x ? nB : nA;
      if (n_mine == 0) continue;
      const int qi = pf3_row(w, x, pair) + r;  // row among the new tokens
      const int qa = c + qi, klen = min(c + len, kcap);  // its key position; keys in total
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n_mine; ++j) {
        const bool got = mbar_wait_bounded(bar_s + 8 * x, ns & 1);
        ++ns;
        if (__any_sync(0xffffffffu, !got) || *abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[NCC][32];
#pragma unroll
        for (int c = 0; c < NCC; ++c)
          tmem_ld32_nowait(tS + lane_off + c * 32, sr[c]);
        tmem_wait_ld();
        const int kb = j * 128;  // key index of the tile's first column
        // whole tile below the diagonal and inside the sequence: no masking
        const bool full = j * 128 + 127 <= qa && j * 128 + 128 <= klen;
        float mxa[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) mxa[a] = -INFINITY;
        if (!full) {
          const int lim = min(qa, klen - 1) - kb;  // last visible column of the row
#pragma unroll
          for (int c = 0; c < NCC; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c * 32 + i > lim) sr[c][i] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int c = 0; c < NCC; ++c)
#pragma unroll
          for (int i = 0; i < 32; i += 2)
            mxa[(i >> 1) & 7] = fmax3(mxa[(i >> 1) & 7], __uint_as_float(sr[c][i]),
                                      __uint_as_float(sr[c][i + 1]));
        float mx = fmax3(fmax3(mxa[0], mxa[1], mxa[2]), fmax3(mxa[3], mxa[4], mxa[5]),
                         fmaxf(mxa[6], mxa[7]));
        mx *= scale_log2;  // scale > 0: max of scaled scores = scaled max
        const bool need = mx > m + kRescaleThreshold;
        float alpha = 1.f;
        if (need) {
          alpha = exp2f(m - mx);
          m = mx;
        }
        const float neg_m = -m;
        // row sum in 4 independent partials of (even, odd) column pairs
        float rsa[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
        // exponentials, row sums and P; `kPoly` (a warp whose rows are all
        // unmasked in this tile) takes exp2_poly2 for the first NB_PF3_POLY
        // of every 8 value pairs
        auto exp_tile = [&](auto poly_tag) {
          constexpr bool kPoly = decltype(poly_tag)::value;
#pragma unroll
          for (int c = 0; c < NCC; ++c) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              uint32_t pk[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                // masked scores are -inf: the MUFU's exp2 gives exactly 0, so
                // tiles with masked rows use it for every value
                const int i = hh * 16 + 2 * e;
                float x0, x1;
                fma_f32x2(x0, x1, __uint_as_float(sr[c][i]), __uint_as_float(sr[c][i + 1]),
                          scale_log2, scale_log2, neg_m, neg_m);
                float p0, p1;
                if (kPoly && e < NB_PF3_POLY) {
                  exp2_poly2(p0, p1, x0, x1);
                } else {
                  p0 = ex2_approx(x0);
                  p1 = ex2_approx(x1);
                }
                add_f32x2(rsa[e & 3][0], rsa[e & 3][1], rsa[e & 3][0], rsa[e & 3][1], p0, p1);
                pk[e] = Mma<T>::pack(p0, p1);
              }
              // P over S's first 64 columns
              tmem_st8(tS + lane_off + c * 16 + hh * 8, pk);
            }
          }
        };
        if (NB_PF3_POLY > 0 && __all_sync(0xffffffffu, full))
          exp_tile(std::true_type{});
        else
          exp_tile(std::false_type{});
        add_f32x2(rsa[0][0], rsa[0][1], rsa[0][0], rsa[0][1], rsa[1][0], rsa[1][1]);
        add_f32x2(rsa[2][0], rsa[2][1], rsa[2][0], rsa[2][1], rsa[3][0], rsa[3][1]);
        const float rs = (rsa[0][0] + rsa[2][0]) + (rsa[0][1] + rsa[2][1]);
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // rescale this thread's O columns (P_X(j-1).V_{j-1} is complete:
          // the commit that signalled S_X(j) covers it; P_X(j).V_j waits for
          // this group's arrivals below)
#pragma unroll 1
          for (int c = 0; c < OC; ++c) {
            float v[32];
            tmem_ld32(tO + lane_off + c * 32, v);
#pragma unroll
            for (int i = 0; i < 32; i += 2) mul_f32x2(v[i], v[i + 1], v[i], v[i + 1], alpha, alpha);
            tmem_st32(tO + lane_off + c * 32, v);
          }
        }
        tmem_wait_st();
        l = l * alpha + rs;
        tc_fence_before();
        mbar_arrive(bar_p + 8 * x);
      }
      if (!ok) break;
      // the row sum to the epilogue warps (double-buffered by unit: the
      // group can finish the next unit before the epilogue read this one)
      const uint32_t up = nunits & 1;
      rowsum[(2 * x + up) * 128 + r] = l;
      mbar_arrive(bar_l + 8 * (2 * x + up));
      ++nunits;
    }
    if (!ok) {
      *abort_flag = 1;
      if (lane == 0) set_error(kErrTimeout);
    }
  } else {
    setmaxnreg_dec<kPf3EpilogueRegs>();
    // ---------------- epilogue: O_X / l -> out rows ----------------
    constexpr int OC = D / 32;  // 32-column O chunks
    const int wq = warp & 3;    // TMEM lane quarter, as in the softmax groups
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const int r = wq * 32 + lane;
    uint32_t ne[2] = {0, 0};    // units written out per tile
    bool ok = true;
    for (int rd = 0, u = unit_of(0); ok && u < n_units; u = unit_of(++rd)) {
      const Pf3Unit w = pf3_unit(u, hq, B, nqb, pair);
      int s0, len, nA, nB, c;
      if (!extent(w, s0, len, nA, nB, c)) continue;
      const int nx[2] = {nA, nB};
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        if (!nx[x]) continue;
        const uint32_t e = ne[x]++;
        const uint32_t lb = 2 * x + (e & 1);
        // O_X final (the MMA warp's commit after the unit's last P.V) and
        // the group's row sums written
        const bool done = mbar_wait_bounded(bar_o + 8 * x, e & 1) &&
                          mbar_wait_bounded(bar_l + 8 * lb, (e >> 1) & 1);
        // one answer for all four epilogue warps (they share named barriers)
        if (named_bar_or(1, 128, !done || *abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float inv = 1.f / rowsum[lb * 128 + r];
        const int q0 = pf3_row(w, x, pair);
        const int qi = q0 + r;  // row among the new tokens
        const uint32_t tO = tmem + (x ? G::kOB : G::kOA);
        if (o_tma && q0 + 128 <= len) {
          // a whole tile inside the sequence: 64-column boxes staged in
          // shared memory (128-byte swizzle: 16-byte chunk k of row r at
          // k ^ (r mod 8)) and written by one TMA store each
          const uint32_t stage = sb + G::kOStage + r * 128;
#pragma unroll 1
          for (int hb = 0; hb < D / 64; ++hb) {
            // the box is free once the previous store has read it
            if (warp == kPf3WarpEpi && lane == 0) bulk_wait_read_all();
            named_bar_sync(1, 128);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              float v[32];
              tmem_ld32(tO + lane_off + (hb * 2 + half) * 32, v);
              if (hb * 2 + half + 1 == OC) {
                tc_fence_before();
                mbar_arrive(bar_ofree + 8 * x);  // O_X read out: the MMA warp may overwrite it
              }
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                uint32_t pk[4];
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                  float a0, a1;
                  mul_f32x2(a0, a1, v[k * 8 + 2 * h], v[k * 8 + 2 * h + 1], inv, inv);
                  pk[h] = Mma<T>::pack(a0, a1);
                }
                const uint32_t chunk = (uint32_t)((half * 4 + k) ^ (r & 7));
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(stage + chunk * 16),
                             "r"(pk[0]), "r"(pk[1]), "r"(pk[2]), "r"(pk[3])
                             : "memory");
              }
            }
            fence_proxy_async_smem();
            named_bar_sync(1, 128);
            if (warp == kPf3WarpEpi && lane == 0) {
              tma_store_2d(&omap, sb + G::kOStage, pf3_head(w, x, pair) * D + hb * 64, s0 + q0);
              bulk_commit_group();
            }
          }
          continue;
        }
        T* dst = out + (int64_t)(s0 + qi) * os + (int64_t)pf3_head(w, x, pair) * D;
        // one 32-column chunk at a time: load, normalise, convert, store
#pragma unroll 1
        for (int cc = 0; cc < OC; ++cc) {
          float v[32];
          tmem_ld32(tO + lane_off + cc * 32, v);
          if (qi < len) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              uint32_t pk[4];
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                float a0, a1;
                mul_f32x2(a0, a1, v[k * 8 + 2 * h], v[k * 8 + 2 * h + 1], inv, inv);
                pk[h] = Mma<T>::pack(a0, a1);
              }
              *reinterpret_cast<uint4*>(dst + cc * 32 + k * 8) =
                  make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(bar_ofree + 8 * x);  // the MMA warp may overwrite O_X
      }
    }
    if (!ok) {
      *abort_flag = 1;
      if (lane == 0) set_error(kErrTimeout);
    }
    // the staged boxes are written out before the CTA exits
    if (warp == kPf3WarpEpi && lane == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kPf3WarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, G::kTmemCols);
  }
}

}  // namespace nb

namespace nbh {

// Head pairs for even GQA groups (NB_PF3_PAIR=0 keeps the row halves of one
// head; diagnostics).
inline int pf3_pair_heads(int group) {
  static int on = [] {
    const char* e = getenv("NB_PF3_PAIR");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return (on && group % 2 == 0) ? 1 : 0;
}

// The kernel's warpgroups re-divide the registers the block is launched
// with (setmaxnreg); a block launched with fewer than the split adds up to
// would leave the softmax warps waiting for registers, so the compiled
// kernel's per-thread count is checked once per instantiation before its
// first launch.
template <typename T, int D>
int pf3_check_registers() {
  static const int rc = [] {
    cudaFuncAttributes a{};
    if (cudaFuncGetAttributes(&a, (const void*)nb::prefill_tc3_kernel<T, D>) != cudaSuccess)
      return fail(NB_ERR_CUDA, "prefill_tc3: cudaFuncGetAttributes failed");
    const long have = (long)a.numRegs * nb::kPf3Threads;
    const long need = 128L * (2 * nb::kPf3SoftmaxRegs + nb::kPf3EpilogueRegs + nb::kPf3IssueRegs);
    if (a.numRegs != nb::kPf3LaunchRegs || have < need)
      return fail(NB_ERR_UNSUPPORTED,
                  "prefill_tc3: compiled with %d registers per thread, the register split "
                  "needs %d",
                  a.numRegs, nb::kPf3LaunchRegs);
    return 0;
  }();
  return rc;
}

// Whole 128-row output tiles go out through shared memory and TMA stores
// (NB_PF3_TMA_STORE=0: every row by plain 16-byte stores; diagnostics).
inline bool pf3_tma_store_enabled() {
  static const bool on = [] {
    const char* e = getenv("NB_PF3_TMA_STORE");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename T, int D>
int launch_prefill_tc3_s(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                         const int32_t* cu, int B, int T_, int hq, int group, int max_seqlen,
                         float sl2, T* out, int64_t os, int dtype, cudaStream_t st,
                         const nb::Pf3Paged& pg) {
  using G = nb::Pf3Geom<D>;
  // the output map (16-byte aligned base and row pitch; otherwise, or when
  // disabled, plain stores and any valid map in its place)
  CUtensorMap om = qm;
  int o_tma = 0;
  if (pf3_tma_store_enabled() && T_ > 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
      ((uint64_t)os * sizeof(T)) % 16 == 0) {
    if (tensor_map_2d(&om, out, dtype, (uint64_t)hq * D, (uint64_t)T_, (uint64_t)os * sizeof(T),
                      64, 128) == NB_OK)
      o_tma = 1;
    else
      om = qm;
  }
  auto kern = nb::prefill_tc3_kernel<T, D>;
  if (int r1 = pf3_check_registers<T, D>()) return r1;
  if (int r2 = ensure_max_smem((const void*)kern, G::kSmem, "prefill_tc3")) return r2;
  const int pair = pf3_pair_heads(group);
  const int nqb = pair ? (max_seqlen + 127) / 128 : (max_seqlen + 255) / 256;
  const int64_t units = (int64_t)nqb * (pair ? hq / 2 : hq) * B;
  if (units > INT32_MAX) return fail(NB_ERR_UNSUPPORTED, "too many prefill work units");
  const int grid = (int)std::min<int64_t>(units, num_sms());
  kern<<<grid, nb::kPf3Threads, G::kSmem, st>>>(qm, km, vm, cu, B, hq, group, nqb, pair, sl2, out,
                                                 os, pg, om, o_tma);
  return check_launch("prefill_tc3");
}

template <typename T, int D>
int launch_prefill_tc3(const void* q, int64_t qs, const void* k, int64_t ks, const void* v,
                       int64_t vs, int hq, int hk, int group, const int32_t* cu, int B, int T_,
                       int max_seqlen, float sl2, void* out, int64_t os, int dtype,
                       cudaStream_t st) {
  CUtensorMap qm, km, vm;
  int rc = tensor_map_2d(&qm, q, dtype, (uint64_t)hq * D, T_, (uint64_t)qs * 2, 64, 128);
  if (!rc) rc = tensor_map_2d(&km, k, dtype, (uint64_t)hk * D, T_, (uint64_t)ks * 2, 64, 128);
  if (!rc) rc = tensor_map_2d(&vm, v, dtype, (uint64_t)hk * D, T_, (uint64_t)vs * 2, 64, 128);
  if (rc) return rc;
  const nb::Pf3Paged pg{nullptr, 0, 0, nullptr, 0, 0};
  return launch_prefill_tc3_s<T, D>(qm, km, vm, cu, B, T_, hq, group, max_seqlen, sl2, (T*)out, os,
                                    dtype, st, pg);
}

// Paged form: q of the new tokens as above; K and V of every key (cached
// prefix + new tokens) from the cache through the block table.
template <typename T, int D>
int launch_prefill_tc3_paged(const void* q, int64_t qs, const void* cache, int nblk, int hk,
                             int hq, int group, const int32_t* bt, int64_t bts, int maxb,
                             const int32_t* ctx, const int32_t* cu, int B, int T_, int max_seqlen,
                             float sl2, void* out, int64_t os, int dtype, cudaStream_t st) {
  CUtensorMap qm, cm;
  int rc = tensor_map_2d(&qm, q, dtype, (uint64_t)hq * D, T_, (uint64_t)qs * 2, 64, 128);
  if (!rc)
    rc = tensor_map_2d(&cm, cache, dtype, (uint64_t)D, (uint64_t)2 * nblk * hk * 16,
                       (uint64_t)D * 2, 64, 16);
  if (rc) return rc;
  const nb::Pf3Paged pg{bt, bts, maxb, ctx, nblk, hk};
  return launch_prefill_tc3_s<T, D>(qm, cm, cm, cu, B, T_, hq, group, max_seqlen, sl2, (T*)out, os,
                                    dtype, st, pg);
}

}  // namespace nbh
