// Causal prefill attention over each sequence's new tokens.
//
// prefill_tc_kernel (below) is the bf16/fp16 path on the 5th-generation
// tensor cores.  prefill_simt_kernel is the fp32 path and the fallback for
// head dims the tensor-core kernel does not take: one warp per (query token,
// query head), a CTA holds 4 consecutive queries of one head so they stream
// the same keys through L1, online softmax in base 2 with shuffle-reduced dot
// products.
#pragma once
#include "nb_common.cuh"

namespace nb {

template <typename T, int D>
__global__ void __launch_bounds__(128)
    prefill_simt_kernel(const T* __restrict__ q, int64_t qs, const T* __restrict__ k, int64_t ks,
                        const T* __restrict__ v, int64_t vs, int hq, int group,
                        const int32_t* __restrict__ cu, float scale_log2, T* __restrict__ out,
                        int64_t os) {
  constexpr int EPL = D / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, head = blockIdx.y;
  const int s0 = __ldg(cu + b), len = __ldg(cu + b + 1) - s0;
  const int i = blockIdx.x * 4 + warp;
  if (i >= len) return;
  const int kh = head / group;
  const int tq = s0 + i;
  float qv[EPL], acc[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    qv[e] = Dt<T>::to_f(q[(int64_t)tq * qs + (int64_t)head * D + lane * EPL + e]);
    acc[e] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int j = 0; j <= i; ++j) {
    const int64_t tk = s0 + j;
    const T* kr = k + tk * ks + (int64_t)kh * D + lane * EPL;
    const T* vr = v + tk * vs + (int64_t)kh * D + lane * EPL;
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) s = fmaf(qv[e], Dt<T>::to_f(kr[e]), s);
    s = warp_sum(s) * scale_log2;
    const float mn = fmaxf(m, s);
    const float al = exp2f(m - mn);
    const float p = exp2f(s - mn);
    l = l * al + p;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = fmaf(acc[e], al, p * Dt<T>::to_f(vr[e]));
    m = mn;
  }
  const float inv = 1.f / l;
#pragma unroll
  for (int e = 0; e < EPL; ++e)
    out[(int64_t)tq * os + (int64_t)head * D + lane * EPL + e] = Dt<T>::from_f(acc[e] * inv);
}


// ---------------------------------------------------------------------------
// Tensor-core prefill (bf16/fp16, head_dim 64/128) on tcgen05 + TMEM.
//
// One CTA of 4 warps per (128-query tile, query head, sequence).  Q, K and V
// tiles (128 rows x 64 columns per 16 KB atom, 128-byte swizzle) arrive by
// TMA; K/V are double-buffered.  Per KV tile j (causal: j = 0..tile):
//   S[128 x 128] = Q . K_j^T        tcgen05.mma into TMEM columns [0, 128)
//   each thread owns one query row (= one TMEM lane): pass 1 over its S row
//   finds the tile max, pass 2 writes P = exp2(s - m) (bf16/fp16, swizzled)
//   to shared memory and sums it
//   O += P . V_j                    tcgen05.mma into TMEM columns [128, 128+D)
// O stays in TMEM for the whole row of tiles.  The running max m is only
// raised when a tile's max exceeds it by more than 8 (log2 units, a factor of
// 256); then the warp rescales its O rows in TMEM (ld, multiply, st).  With a
// stale m every p is at most 2^8, far inside fp32/bf16 range, and O / l is
// exact, so the lazy update changes no result but skips almost all
// rescaling.  The P.V MMA of tile j runs while the S MMA and the max pass of
// tile j+1 proceed.  One thread issues the MMAs and TMA loads and commits the
// MMAs to mbarriers; every wait is bounded.
// ---------------------------------------------------------------------------
template <int D> struct PfGeom {
  static constexpr int kAtom = 128 * 128;            // 128 rows x 128 B
  static constexpr int kTile = (D / 64) * kAtom;     // one Q, K or V tile
  static constexpr int kQ = 0;
  static constexpr int kK = kTile;                   // 2 stages
  static constexpr int kV = kK + 2 * kTile;          // 2 stages
  static constexpr int kP = kV + 2 * kTile;          // 128 x 128 probabilities
  static constexpr int kBars = kP + 2 * kAtom;
  static constexpr int kSmem = kBars + 64 + 1024;
  static constexpr uint32_t kTmemCols = 256;         // S: 128 columns, O: D columns
};

constexpr float kRescaleThreshold = 8.0f;

template <typename T, int D>
__global__ void __launch_bounds__(128, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                      const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const int32_t* __restrict__ cu,
                      int group, float scale_log2, T* __restrict__ out, int64_t os) {
  using G = PfGeom<D>;
  constexpr bool kBf16 = !__is_same(T, __half);
  constexpr uint32_t kIdS = idesc_f16_f32(kBf16, 128, 128, false, false);
  constexpr uint32_t kIdO = idesc_f16_f32(kBf16, 128, D, false, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int s0 = __ldg(cu + b), len = __ldg(cu + b + 1) - s0;
  const int q0 = qt * 128;
  if (q0 >= len) return;
  const int kh = h / group;
  const int n_kv = qt + 1;
  const uint32_t sb = smem_u32(smem);
  const uint32_t bar_q = sb + G::kBars, bar_s = bar_q + 8, bar_o = bar_q + 16;
  const uint32_t bar_kv0 = bar_q + 24;  // + 8 * stage
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::kBars + 48);

  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), G::kTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    mbar_init(bar_q, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    mbar_init(bar_kv0, 1);
    mbar_init(bar_kv0 + 8, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;

  auto load_kv = [&](int j) {  // thread 0 only
    const int st = j & 1;
    const uint32_t bar = bar_kv0 + 8 * st;
    mbar_arrive_expect_tx(bar, 2 * G::kTile);
#pragma unroll
    for (int a = 0; a < D / 64; ++a) {
      tma_load_2d(sb + G::kK + st * G::kTile + a * G::kAtom, &kmap, kh * D + a * 64,
                  s0 + j * 128, bar);
      tma_load_2d(sb + G::kV + st * G::kTile + a * G::kAtom, &vmap, kh * D + a * 64,
                  s0 + j * 128, bar);
    }
  };
  if (tid == 0) {
    mbar_arrive_expect_tx(bar_q, G::kTile);
#pragma unroll
    for (int a = 0; a < D / 64; ++a)
      tma_load_2d(sb + G::kQ + a * G::kAtom, &qmap, h * D + a * 64, s0 + q0, bar_q);
    load_kv(0);
    if (n_kv > 1) load_kv(1);
  }

  const int r = warp * 32 + lane;  // query row of this thread = TMEM lane
  const int qi = q0 + r;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  float m = -INFINITY, l = 0.f;
  bool failed = false;

  for (int j = 0; j < n_kv; ++j) {
    const int st = j & 1;
    if (tid == 0) {
      bool w = j > 0 || mbar_wait_bounded(bar_q, 0);
      w = w && mbar_wait_bounded(bar_kv0 + 8 * st, (j >> 1) & 1);
      if (w) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * G::kAtom + (kk & 3) * 32;
          tc_mma_f16_ss(tS, smem_desc_sw128(sb + G::kQ + off, 16, 1024),
                        smem_desc_sw128(sb + G::kK + st * G::kTile + off, 16, 1024), kIdS,
                        kk > 0);
        }
        tc_commit(bar_s);
      }
    }
    if (__syncthreads_or(!mbar_wait_bounded(bar_s, j & 1))) { failed = true; break; }
    tc_fence_after();

    // pass 1: this tile's row max of the scaled, masked scores
    const int kb = j * 128;
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float v[32];
      tmem_ld32(tS + lane_off + c * 32, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int col = kb + c * 32 + i;
        if (col <= qi && col < len) mx = fmaxf(mx, v[i] * scale_log2);
      }
    }
    // P.V of the previous tile must be done before P is overwritten, O is
    // rescaled or its V stage is refilled.
    if (j > 0) {
      if (__syncthreads_or(!mbar_wait_bounded(bar_o, (j - 1) & 1))) { failed = true; break; }
      tc_fence_after();
      if (tid == 0 && j + 1 < n_kv) load_kv(j + 1);
    }
    const bool need = mx > m + kRescaleThreshold;  // also true on the first valid tile
    float alpha = 1.f;
    if (need) {
      alpha = exp2f(m - mx);  // 0 when m is still -inf
      m = mx;
    }
    // pass 2: probabilities into the swizzled P tile, row sum
    float rs = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float v[32];
      tmem_ld32(tS + lane_off + c * 32, v);
#pragma unroll
      for (int k = 0; k < 4; ++k) {  // 4 chunks of 8 columns
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i0 = k * 8 + 2 * e;
          const int col = kb + c * 32 + i0;
          const float p0 = (col <= qi && col < len) ? exp2f(v[i0] * scale_log2 - m) : 0.f;
          const float p1 =
              (col + 1 <= qi && col + 1 < len) ? exp2f(v[i0 + 1] * scale_log2 - m) : 0.f;
          rs += p0 + p1;
          pk[e] = Mma<T>::pack(p0, p1);
        }
        const int cc = c * 4 + k;  // 16-byte chunk index 0..15 along the 128 columns
        const uint32_t addr =
            G::kP + (cc >> 3) * G::kAtom + r * 128 + (((cc & 7) ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(smem + addr) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
    l = l * alpha + rs;
    // rescale this warp's O rows in TMEM when any of its rows raised m
    if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        tmem_ld32(tO + lane_off + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= alpha;
        tmem_st32(tO + lane_off + c * 32, v);
      }
      tmem_wait_st();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t aoff = (kk >> 2) * G::kAtom + (kk & 3) * 32;
        tc_mma_f16_ss(tO, smem_desc_sw128(sb + G::kP + aoff, 16, 1024),
                      smem_desc_sw128(sb + G::kV + st * G::kTile + kk * 16 * 128, G::kAtom, 1024),
                      kIdO, (j > 0 || kk > 0) ? 1u : 0u);
      }
      tc_commit(bar_o);
    }
  }
  if (!failed && __syncthreads_or(!mbar_wait_bounded(bar_o, (n_kv - 1) & 1))) failed = true;

  if (failed) {
    if (tid == 0) set_error(kErrTimeout);
  } else {
    tc_fence_after();
    const float inv = 1.f / l;
    T* dst = out + (int64_t)(s0 + qi) * os + (int64_t)h * D;
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      float v[32];
      tmem_ld32(tO + lane_off + c * 32, v);
      if (qi < len) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            pk[e] = Mma<T>::pack(v[k * 8 + 2 * e] * inv, v[k * 8 + 2 * e + 1] * inv);
          *reinterpret_cast<uint4*>(dst + c * 32 + k * 8) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, G::kTmemCols);
  }
}


// ---------------------------------------------------------------------------
// Tensor-core prefill, warp-specialised (bf16/fp16, head_dim 64/128).
//
// One CTA per (256 query rows, query head, sequence) holding two 128-row Q
// tiles, A and B, that share every K/V tile.  Nine warps:
//   warps 0-3  softmax for tile A (thread = query row = TMEM lane)
//   warps 4-7  softmax for tile B
//   warp 8     TMA producer and tcgen05 MMA issuer (lane 0)
// Tensor memory (512 columns): S_A [0,128), S_B [128,256), O_A [256, 256+D),
// O_B [256+D, 256+2D).  Per KV tile j the issuer runs S_A = Q_A K_j^T and
// S_B = Q_B K_j^T back to back; while the tensor core works on S_B, the A
// warps turn S_A into probabilities and write them as bf16/fp16 pairs back
// over S_A's first 64 columns (tcgen05.st); the issuer then runs
// O_A += P_A V_j with P_A read straight from tensor memory, and the same for
// B.  So the two softmax groups and the tensor core take turns instead of
// waiting for each other, no P tile goes through shared memory, and the
// only shared-memory traffic is TMA-loaded Q, K and V (2-stage K/V ring).
// The running max is raised lazily as in prefill_tc_kernel.  The commit
// that signals S_X(j) also covers O_X += P_X V_{j-1}, so a softmax group may
// rescale its O rows as soon as it sees S_X(j).  Every wait is bounded and
// an abort flag lets all roles leave together.
// ---------------------------------------------------------------------------
template <int D> struct Pf2Geom {
  static constexpr int kAtom = 128 * 128;
  static constexpr int kTile = (D / 64) * kAtom;
  static constexpr int kQA = 0;
  static constexpr int kQB = kTile;
  static constexpr int kK = 2 * kTile;          // 2 stages
  static constexpr int kV = kK + 2 * kTile;     // 2 stages
  static constexpr int kBars = kV + 2 * kTile;
  static constexpr int kSmem = kBars + 128 + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kSA = 0, kSB = 128, kOA = 256, kOB = 256 + D;
};

template <typename T, int D>
__global__ void __launch_bounds__(288, 1)
    prefill_tc2_kernel(const __grid_constant__ CUtensorMap qmap,
                       const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap, const int32_t* __restrict__ cu,
                       int group, float scale_log2, T* __restrict__ out, int64_t os) {
  using G = Pf2Geom<D>;
  constexpr bool kBf16 = !__is_same(T, __half);
  constexpr uint32_t kIdS = idesc_f16_f32(kBf16, 128, 128, false, false);
  constexpr uint32_t kIdO = idesc_f16_f32(kBf16, 128, D, false, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int s0 = __ldg(cu + b), len = __ldg(cu + b + 1) - s0;
  const int q0 = qt * 256;
  if (q0 >= len) return;
  const bool hasB = q0 + 128 < len;
  const int nA = 2 * qt + 1;                 // KV tiles under tile A's rows (causal)
  const int nB = hasB ? 2 * qt + 2 : 0;
  const int n_kv = hasB ? nB : nA;
  const int kh = h / group;
  const uint32_t sb = smem_u32(smem);
  // barriers: q, kv[2], kvfree[2], sA, sB, pA, pB, done
  const uint32_t bar_q = sb + G::kBars;
  const uint32_t bar_kv = bar_q + 8, bar_free = bar_q + 24;
  const uint32_t bar_sA = bar_q + 40, bar_sB = bar_q + 48;
  const uint32_t bar_pA = bar_q + 56, bar_pB = bar_q + 64, bar_done = bar_q + 72;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + G::kBars + 96);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::kBars + 104);

  if (warp == 8) {
    tmem_alloc(smem_u32(tmem_slot), G::kTmemCols);
    tmem_relinquish();
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      mbar_init(bar_q, 1);
      mbar_init(bar_kv, 1);
      mbar_init(bar_kv + 8, 1);
      mbar_init(bar_free, 1);
      mbar_init(bar_free + 8, 1);
      mbar_init(bar_sA, 1);
      mbar_init(bar_sB, 1);
      mbar_init(bar_pA, 128);
      mbar_init(bar_pB, 128);
      mbar_init(bar_done, 1);
      *abort_flag = 0;
      fence_mbar_init();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (lane == 0) {
      // ---------------- producer + MMA issuer ----------------
      auto fail_out = [&]() { *abort_flag = 1; set_error(kErrTimeout); };
      auto load_kv = [&](int j) {
        const int st = j & 1;
        mbar_arrive_expect_tx(bar_kv + 8 * st, 2 * G::kTile);
#pragma unroll
        for (int a = 0; a < D / 64; ++a) {
          tma_load_2d(sb + G::kK + st * G::kTile + a * G::kAtom, &kmap, kh * D + a * 64,
                      s0 + j * 128, bar_kv + 8 * st);
          tma_load_2d(sb + G::kV + st * G::kTile + a * G::kAtom, &vmap, kh * D + a * 64,
                      s0 + j * 128, bar_kv + 8 * st);
        }
      };
      mbar_arrive_expect_tx(bar_q, (hasB ? 2 : 1) * G::kTile);
#pragma unroll
      for (int a = 0; a < D / 64; ++a) {
        tma_load_2d(sb + G::kQA + a * G::kAtom, &qmap, h * D + a * 64, s0 + q0, bar_q);
        if (hasB) tma_load_2d(sb + G::kQB + a * G::kAtom, &qmap, h * D + a * 64, s0 + q0 + 128, bar_q);
      }
      load_kv(0);
      if (n_kv > 1) load_kv(1);
      // Issue order: S_A(0) S_B(0) | PV_A(0) S_A(1) PV_B(0) S_B(1) | PV_A(1) S_A(2) ...
      // so that group A's softmax of tile j+1 overlaps group B's softmax of
      // tile j and the tensor core's P_B.V_j.
      int kv_ready = -1;  // highest KV tile whose load has been waited for
      auto wait_kv = [&](int j) -> bool {
        if (j <= kv_ready) return true;
        if (!mbar_wait_bounded(bar_kv + 8 * (j & 1), (j >> 1) & 1)) return false;
        kv_ready = j;
        tc_fence_after();
        return true;
      };
      auto issue_s = [&](int j, uint32_t q_off, uint32_t t_col, uint32_t bar) {
        const uint32_t kst = sb + G::kK + (j & 1) * G::kTile;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * G::kAtom + (kk & 3) * 32;
          tc_mma_f16_ss(tmem + t_col, smem_desc_sw128(sb + q_off + off, 16, 1024),
                        smem_desc_sw128(kst + off, 16, 1024), kIdS, kk > 0);
        }
        tc_commit(bar);
      };
      auto issue_pv = [&](int j, uint32_t s_col, uint32_t o_col) {
        const uint32_t vst = sb + G::kV + (j & 1) * G::kTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16_ts(tmem + o_col, tmem + s_col + kk * 8,
                        smem_desc_sw128(vst + kk * 16 * 128, G::kAtom, 1024), kIdO,
                        (j > 0 || kk > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait_bounded(bar_q, 0) && wait_kv(0);
      if (ok) {
        tc_fence_after();
        issue_s(0, G::kQA, G::kSA, bar_sA);
        if (hasB) issue_s(0, G::kQB, G::kSB, bar_sB);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int st = j & 1;
        if (j < nA) {
          if (!mbar_wait_bounded(bar_pA, j & 1) || *abort_flag) { ok = false; break; }
          tc_fence_after();
          issue_pv(j, G::kSA, G::kOA);
          if (j + 1 < nA) {
            if (!wait_kv(j + 1)) { ok = false; break; }
            issue_s(j + 1, G::kQA, G::kSA, bar_sA);
          }
        }
        if (j < nB) {
          if (!mbar_wait_bounded(bar_pB, j & 1) || *abort_flag) { ok = false; break; }
          tc_fence_after();
          issue_pv(j, G::kSB, G::kOB);
          if (j + 1 < nB) {
            if (!wait_kv(j + 1)) { ok = false; break; }
            issue_s(j + 1, G::kQB, G::kSB, bar_sB);
          }
        }
        tc_commit(bar_free + 8 * st);
        // refill this stage with tile j+2 once tile j's MMAs have released it
        if (j + 2 < n_kv) {
          if (!mbar_wait_bounded(bar_free + 8 * st, (j >> 1) & 1)) { ok = false; break; }
          load_kv(j + 2);
        }
      }
      if (!ok) fail_out();
      tc_commit(bar_done);
    }
  } else {
    // ---------------- softmax groups ----------------
    const int wg = warp >> 2;  // 0 = tile A, 1 = tile B
    const int n_mine = wg ? nB : nA;
    const uint32_t tSx = tmem + (wg ? G::kSB : G::kSA);
    const uint32_t tOx = tmem + (wg ? G::kOB : G::kOA);
    const uint32_t bar_s = wg ? bar_sB : bar_sA;
    const uint32_t bar_p = wg ? bar_pB : bar_pA;
    const int r = (warp & 3) * 32 + lane;
    const int qi = q0 + wg * 128 + r;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < n_mine; ++j) {
      const bool got = mbar_wait_bounded(bar_s, j & 1);
      if (__any_sync(0xffffffffu, !got) || *abort_flag) { *abort_flag = 1; break; }
      tc_fence_after();
      const int kb = j * 128;
      // whole tile below the diagonal and inside the sequence: no masking
      const bool full = kb + 127 <= qi && kb + 128 <= len;
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(tSx + lane_off + c * 32, v);
        if (full) {
#pragma unroll
          for (int i = 0; i < 32; ++i) mx = fmaxf(mx, v[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int col = kb + c * 32 + i;
            mx = fmaxf(mx, (col <= qi && col < len) ? v[i] : -INFINITY);
          }
        }
      }
      mx *= scale_log2;  // scale > 0: max of scaled scores = scaled max
      const bool need = mx > m + kRescaleThreshold;
      float alpha = 1.f;
      if (need) {
        alpha = exp2f(m - mx);
        m = mx;
      }
      if (j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          float v[32];
          tmem_ld32(tOx + lane_off + c * 32, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tmem_st32(tOx + lane_off + c * 32, v);
        }
      }
      const float neg_m = -m;
      float rs = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(tSx + lane_off + c * 32, v);
        uint32_t pk[16];
        if (full) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float p0 = ex2_approx(fmaf(v[2 * e], scale_log2, neg_m));
            const float p1 = ex2_approx(fmaf(v[2 * e + 1], scale_log2, neg_m));
            rs += p0 + p1;
            pk[e] = Mma<T>::pack(p0, p1);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int col = kb + c * 32 + 2 * e;
            const float p0 = (col <= qi && col < len) ? ex2_approx(fmaf(v[2 * e], scale_log2, neg_m)) : 0.f;
            const float p1 = (col + 1 <= qi && col + 1 < len)
                                 ? ex2_approx(fmaf(v[2 * e + 1], scale_log2, neg_m)) : 0.f;
            rs += p0 + p1;
            pk[e] = Mma<T>::pack(p0, p1);
          }
        }
        tmem_st16(tSx + lane_off + c * 16, pk);  // P over S's first 64 columns
      }
      tmem_wait_st();
      l = l * alpha + rs;
      tc_fence_before();
      mbar_arrive(bar_p);
    }
    const bool done = mbar_wait_bounded(bar_done, 0);
    if (n_mine > 0 && done && !*abort_flag) {
      tc_fence_after();
      const float inv = 1.f / l;
      T* dst = out + (int64_t)(s0 + qi) * os + (int64_t)h * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        tmem_ld32(tOx + lane_off + c * 32, v);
        if (qi < len) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint32_t pk[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              pk[e] = Mma<T>::pack(v[k * 8 + 2 * e] * inv, v[k * 8 + 2 * e + 1] * inv);
            *reinterpret_cast<uint4*>(dst + c * 32 + k * 8) =
                make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, G::kTmemCols);
  }
}

}  // namespace nb

namespace nbh {

template <typename T, int D>
int launch_prefill_simt(const void* q, int64_t qs, const void* k, int64_t ks, const void* v,
                        int64_t vs, int hq, int group, const int32_t* cu, int B, int max_seqlen,
                        float sl2, void* out, int64_t os, cudaStream_t st) {
  dim3 grid((max_seqlen + 3) / 4, hq, B);
  nb::prefill_simt_kernel<T, D><<<grid, 128, 0, st>>>((const T*)q, qs, (const T*)k, ks,
                                                      (const T*)v, vs, hq, group, cu, sl2,
                                                      (T*)out, os);
  return check_launch("prefill_simt");
}


template <typename T, int D>
int launch_prefill_tc(const void* q, int64_t qs, const void* k, int64_t ks, const void* v,
                      int64_t vs, int hq, int hk, int group, const int32_t* cu, int B, int T_,
                      int max_seqlen, float sl2, void* out, int64_t os, int dtype,
                      cudaStream_t st) {
  using G = nb::PfGeom<D>;
  CUtensorMap qm, km, vm;
  int rc = tensor_map_2d(&qm, q, dtype, (uint64_t)hq * D, T_, (uint64_t)qs * 2, 64, 128);
  if (!rc) rc = tensor_map_2d(&km, k, dtype, (uint64_t)hk * D, T_, (uint64_t)ks * 2, 64, 128);
  if (!rc) rc = tensor_map_2d(&vm, v, dtype, (uint64_t)hk * D, T_, (uint64_t)vs * 2, 64, 128);
  if (rc) return rc;
  auto kern = nb::prefill_tc_kernel<T, D>;
  if (int r2 = ensure_max_smem((const void*)kern, G::kSmem, "prefill_tc")) return r2;
  dim3 grid((max_seqlen + 127) / 128, hq, B);
  kern<<<grid, 128, G::kSmem, st>>>(qm, km, vm, cu, group, sl2, (T*)out, os);
  return check_launch("prefill_tc");
}


template <typename T, int D>
int launch_prefill_tc2(const void* q, int64_t qs, const void* k, int64_t ks, const void* v,
                       int64_t vs, int hq, int hk, int group, const int32_t* cu, int B, int T_,
                       int max_seqlen, float sl2, void* out, int64_t os, int dtype,
                       cudaStream_t st) {
  using G = nb::Pf2Geom<D>;
  CUtensorMap qm, km, vm;
  int rc = tensor_map_2d(&qm, q, dtype, (uint64_t)hq * D, T_, (uint64_t)qs * 2, 64, 128);
  if (!rc) rc = tensor_map_2d(&km, k, dtype, (uint64_t)hk * D, T_, (uint64_t)ks * 2, 64, 128);
  if (!rc) rc = tensor_map_2d(&vm, v, dtype, (uint64_t)hk * D, T_, (uint64_t)vs * 2, 64, 128);
  if (rc) return rc;
  auto kern = nb::prefill_tc2_kernel<T, D>;
  if (int r2 = ensure_max_smem((const void*)kern, G::kSmem, "prefill_tc2")) return r2;
  dim3 grid((max_seqlen + 255) / 256, hq, B);
  kern<<<grid, 288, G::kSmem, st>>>(qm, km, vm, cu, group, sl2, (T*)out, os);
  return check_launch("prefill_tc2");
}

inline int prefill_version() {
  static int v = [] {
    // "1": single-group kernel, "2": per-unit two-group kernel (diagnostics);
    // default: the persistent kernel (prefill3.cuh)
    const char* e = getenv("NB_PREFILL_V");
    return (e && e[0] == '1') ? 1 : (e && e[0] == '2') ? 2 : 3;
  }();
  return v;
}

inline bool prefill_tc_enabled() {
  static int on = [] {
    const char* e = getenv("NB_PREFILL_TC");  // "0" forces the SIMT kernel (diagnostics)
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return on != 0;
}

template <typename T>
int launch_prefill_simt_d(int D, const void* q, int64_t qs, const void* k, int64_t ks,
                          const void* v, int64_t vs, int hq, int group, const int32_t* cu, int B,
                          int msl, float sl2, void* out, int64_t os, cudaStream_t st) {
  switch (D) {
    case 32: return launch_prefill_simt<T, 32>(q, qs, k, ks, v, vs, hq, group, cu, B, msl, sl2, out, os, st);
    case 64: return launch_prefill_simt<T, 64>(q, qs, k, ks, v, vs, hq, group, cu, B, msl, sl2, out, os, st);
    case 96: return launch_prefill_simt<T, 96>(q, qs, k, ks, v, vs, hq, group, cu, B, msl, sl2, out, os, st);
    case 128: return launch_prefill_simt<T, 128>(q, qs, k, ks, v, vs, hq, group, cu, B, msl, sl2, out, os, st);
    case 256: return launch_prefill_simt<T, 256>(q, qs, k, ks, v, vs, hq, group, cu, B, msl, sl2, out, os, st);
    default: return fail(NB_ERR_UNSUPPORTED, "head_dim %d not supported by prefill", D);
  }
}

}  // namespace nbh

#include "prefill3.cuh"

extern "C" {

int nb_prefill_attention(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                         const void* v, int64_t v_stride, int num_q_heads, int num_kv_heads,
                         int head_dim, const int32_t* cu_seqlens, int num_seqs, int num_tokens,
                         int max_seqlen, float scale, void* out, int64_t out_stride, int dtype,
                         void* stream) {
  using namespace nbh;
  if (!valid_dtype(dtype)) return fail(NB_ERR_INVALID_ARG, "invalid dtype %d", dtype);
  if (!q || !k || !v || !cu_seqlens || !out) return fail(NB_ERR_INVALID_ARG, "null pointer");
  if (num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || num_seqs < 0 || num_tokens < 0)
    return fail(NB_ERR_INVALID_ARG, "bad sizes");
  if (num_q_heads % num_kv_heads)
    return fail(NB_ERR_INVALID_ARG, "num_q_heads not a multiple of num_kv_heads");
  if (q_stride < (int64_t)num_q_heads * head_dim || k_stride < (int64_t)num_kv_heads * head_dim ||
      v_stride < (int64_t)num_kv_heads * head_dim || out_stride < (int64_t)num_q_heads * head_dim)
    return fail(NB_ERR_INVALID_ARG, "row stride too small");
  if (num_seqs == 0 || num_tokens == 0) return NB_OK;
  if (max_seqlen <= 0) return fail(NB_ERR_INVALID_ARG, "max_seqlen must be > 0");
  const int group = num_q_heads / num_kv_heads;
  const float sl2 = scale * nb::kLog2e;
  cudaStream_t st = (cudaStream_t)stream;
  const bool tc = dtype != NB_DTYPE_F32 && (head_dim == 64 || head_dim == 128) &&
                  prefill_tc_enabled() && (q_stride * 2) % 16 == 0 && (k_stride * 2) % 16 == 0 &&
                  (v_stride * 2) % 16 == 0 && (out_stride * 2) % 16 == 0 &&
                  (uintptr_t)q % 16 == 0 && (uintptr_t)k % 16 == 0 && (uintptr_t)v % 16 == 0 &&
                  (uintptr_t)out % 16 == 0;
  if (tc) {
#define NB_ARGS q, q_stride, k, k_stride, v, v_stride, num_q_heads, num_kv_heads, group,         \
                cu_seqlens, num_seqs, num_tokens, max_seqlen, sl2, out, out_stride, dtype, st
    if (prefill_version() == 3) {
      if (dtype == NB_DTYPE_BF16)
        return head_dim == 64 ? launch_prefill_tc3<__nv_bfloat16, 64>(NB_ARGS)
                              : launch_prefill_tc3<__nv_bfloat16, 128>(NB_ARGS);
      return head_dim == 64 ? launch_prefill_tc3<__half, 64>(NB_ARGS)
                            : launch_prefill_tc3<__half, 128>(NB_ARGS);
    }
    if (prefill_version() == 2) {
      if (dtype == NB_DTYPE_BF16)
        return head_dim == 64 ? launch_prefill_tc2<__nv_bfloat16, 64>(NB_ARGS)
                              : launch_prefill_tc2<__nv_bfloat16, 128>(NB_ARGS);
      return head_dim == 64 ? launch_prefill_tc2<__half, 64>(NB_ARGS)
                            : launch_prefill_tc2<__half, 128>(NB_ARGS);
    }
    if (dtype == NB_DTYPE_BF16)
      return head_dim == 64 ? launch_prefill_tc<__nv_bfloat16, 64>(NB_ARGS)
                            : launch_prefill_tc<__nv_bfloat16, 128>(NB_ARGS);
    return head_dim == 64 ? launch_prefill_tc<__half, 64>(NB_ARGS)
                          : launch_prefill_tc<__half, 128>(NB_ARGS);
#undef NB_ARGS
  }
  switch (dtype) {
    case NB_DTYPE_F32: return launch_prefill_simt_d<float>(head_dim, q, q_stride, k, k_stride, v, v_stride, num_q_heads, group, cu_seqlens, num_seqs, max_seqlen, sl2, out, out_stride, st);
    case NB_DTYPE_F16: return launch_prefill_simt_d<__half>(head_dim, q, q_stride, k, k_stride, v, v_stride, num_q_heads, group, cu_seqlens, num_seqs, max_seqlen, sl2, out, out_stride, st);
    default: return launch_prefill_simt_d<__nv_bfloat16>(head_dim, q, q_stride, k, k_stride, v, v_stride, num_q_heads, group, cu_seqlens, num_seqs, max_seqlen, sl2, out, out_stride, st);
  }
}

int nb_prefill_attention_paged(const void* q, int64_t q_stride, const void* kv_cache,
                               int num_blocks, int num_kv_heads, const int32_t* block_table,
                               int64_t bt_stride, int max_blocks, const int32_t* context_lens,
                               int num_q_heads, int head_dim, const int32_t* cu_seqlens,
                               int num_seqs, int num_tokens, int max_seqlen, float scale,
                               void* out, int64_t out_stride, int dtype, void* stream) {
  using namespace nbh;
  if (dtype != NB_DTYPE_BF16 && dtype != NB_DTYPE_F16)
    return fail(NB_ERR_UNSUPPORTED, "paged prefill takes bf16 or fp16");
  if (head_dim != 64 && head_dim != 128)
    return fail(NB_ERR_UNSUPPORTED, "paged prefill takes head_dim 64 or 128 (got %d)", head_dim);
  if (!q || !kv_cache || !block_table || !context_lens || !cu_seqlens || !out)
    return fail(NB_ERR_INVALID_ARG, "null pointer");
  if (num_q_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 || max_blocks <= 0 ||
      num_seqs < 0 || num_tokens < 0 || bt_stride < max_blocks)
    return fail(NB_ERR_INVALID_ARG, "bad sizes");
  if (num_q_heads % num_kv_heads)
    return fail(NB_ERR_INVALID_ARG, "num_q_heads not a multiple of num_kv_heads");
  if (q_stride < (int64_t)num_q_heads * head_dim || out_stride < (int64_t)num_q_heads * head_dim)
    return fail(NB_ERR_INVALID_ARG, "row stride too small");
  if ((int64_t)2 * num_blocks * num_kv_heads * 16 > INT32_MAX)
    return fail(NB_ERR_UNSUPPORTED, "cache rows exceed int32");
  if (num_seqs == 0 || num_tokens == 0) return NB_OK;
  if (max_seqlen <= 0) return fail(NB_ERR_INVALID_ARG, "max_seqlen must be > 0");
  if ((q_stride * 2) % 16 || (out_stride * 2) % 16 || (uintptr_t)q % 16 || (uintptr_t)out % 16 ||
      (uintptr_t)kv_cache % 16)
    return fail(NB_ERR_UNSUPPORTED, "paged prefill needs 16-byte aligned rows");
  const int group = num_q_heads / num_kv_heads;
  const float sl2 = scale * nb::kLog2e;
  cudaStream_t st = (cudaStream_t)stream;
#define NB_PARGS q, q_stride, kv_cache, num_blocks, num_kv_heads, num_q_heads, group, block_table, \
                 bt_stride, max_blocks, context_lens, cu_seqlens, num_seqs, num_tokens,         \
                 max_seqlen, sl2, out, out_stride, dtype, st
  if (dtype == NB_DTYPE_BF16)
    return head_dim == 64 ? launch_prefill_tc3_paged<__nv_bfloat16, 64>(NB_PARGS)
                          : launch_prefill_tc3_paged<__nv_bfloat16, 128>(NB_PARGS);
  return head_dim == 64 ? launch_prefill_tc3_paged<__half, 64>(NB_PARGS)
                        : launch_prefill_tc3_paged<__half, 128>(NB_PARGS);
#undef NB_PARGS
}

}  // extern "C"
