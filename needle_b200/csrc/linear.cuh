// Dense projection of a decode step on tcgen05: y[M, N] = x[M, K] . W[N, K]^T
// (+ bias[N]) for M <= 256 rows, bf16 / fp16 in, fp32 accumulation, output in
// the input type.  Replaces the torch F.linear calls of needle's
// ColumnParallelLinear / RowParallelLinear / QKV / gate-up / lm_head
// (needle/layers/linear.py:21-98) when the batch is a decode step; the model
// routes only the LM head here (the shape where it measures faster than
// cuBLAS).
//
// At M <= 256 the GEMM sits at the ridge of the roofline (M FLOPs per weight
// byte: 256 against ~255 FLOP/B), and a 128-row weight tile per CTA gives
// only N / 128 tiles (qkv of Llama-3-8B: 48; o_proj and down: 32), far fewer
// than the 148 SMs that must stream the weights.  So:
//
//   * swap-AB: the MMA's M is 128 weight rows (A = W tile, K-major, 128-byte
//     swizzled, as TMA writes it) and its N is the padded token count
//     NT = round_up(M, 32) (B = x tile, K-major); the accumulator is
//     128 lanes (output features) x NT columns (tokens) of tensor memory;
//   * S > 1: the K range of a tile is split over the S CTAs of a thread-block
//     cluster, and their partial accumulators are reduce-scattered through
//     distributed shared memory: 32-column chunk c of the tile belongs to
//     CTA c % S, every CTA pushes the chunks it does not own into the
//     owner's shared memory (the freed pipeline stages), and each owner adds
//     the other partials to its own in rank order and writes its chunks of y
//     (a fixed order: the result is the same on every run; one tile per
//     cluster);
//   * S = 1: persistent CTAs over tiles.  The default tile is 256 weight
//     rows (two 128-row sub-tiles, two accumulators of all 512 TMEM columns)
//     sharing each x tile, so the x share of every stage (x is re-read from
//     L2 by every CTA) is a half instead of two thirds.  With 128-row tiles
//     the two accumulator sets double-buffer instead, so the epilogue of one
//     tile overlaps the next tile.
//   The cluster split-K path (128-row tiles) is kept for shapes with few
//   tiles, selected explicitly: a cluster of S CTAs must be co-resident, and
//   the number of co-resident clusters (45 clusters of 3 at 197 KB of shared
//   memory on a B200) caps it below one tile per cluster for the projections
//   measured here; callers route those shapes to their library GEMM.
//
// Roles (192 threads): warp 0 TMA producer (one lane), warp 1 MMA issuer (one
// lane), warps 2-5 epilogue (warp w reaches TMEM lanes 32 (w % 4) ..: the four
// warps cover the 128 lanes).  Every wait is bounded: a wait that gives up
// sets the timeout bit and a shared abort flag, the roles leave their loops,
// the producer waits (bounded) for its copies in flight and the MMA warp for
// its MMAs, and the cluster's CTAs meet at one final cluster barrier before
// any of them exits, so no CTA's shared memory is written after it left.
#pragma once
#include <algorithm>
#include <cstdlib>

#include "nb_common.cuh"

namespace nb {

constexpr int kLinW = 128 * 128;   // one 128-row weight sub-tile x 64 K x 2 B
constexpr int kLinX = 256 * 128;   // up to 256 token rows x 64 K x 2 B
// Pipeline depth: 4 stages of one sub-tile + x (48 KB), or 3 stages of two
// sub-tiles + x (64 KB); 192 KB either way.
template <int TW> constexpr int lin_stages() { return TW == 2 ? 3 : 4; }
template <int TW> constexpr int lin_stage_bytes() { return TW * kLinW + kLinX; }
constexpr int kLinBars = 192 * 1024;
constexpr int kLinSmem = kLinBars + 256 + 1024;
constexpr int kLinThreads = 192;
constexpr int kLinChunk = 128 * 32 * 4;  // one 32-column chunk of a partial: 16 KB

// TW: 128-row weight sub-tiles per tile (1 or 2; a tile is 128 TW output
// features).  S: CTAs per cluster splitting K (S > 1 only with TW = 1).
template <typename T, int S, int TW>
__global__ void __launch_bounds__(kLinThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap wmap,
                     const __grid_constant__ CUtensorMap xmap, T* __restrict__ y, int64_t ldy,
                     const T* __restrict__ bias, int M, int N, int NT, int n_tiles, int KB) {
  static_assert(S == 1 || TW == 1, "the cluster split takes one sub-tile per tile");
  constexpr bool kBf16 = !__is_same(T, __half);
  constexpr int kStages = lin_stages<TW>();
  constexpr int kStage = lin_stage_bytes<TW>();
  // accumulator sets: two (double buffering) when a tile's accumulators fit
  // twice in tensor memory, else one
  constexpr int kNbuf = (S == 1 && TW == 1) ? 2 : 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sb = smem_u32(smem);
  const uint32_t bar_full = sb + kLinBars;        // [4] stage landed
  const uint32_t bar_empty = bar_full + 32;       // [4] stage read by its MMAs
  const uint32_t bar_acc = bar_full + 64;         // [2] accumulator set final
  const uint32_t bar_accfree = bar_full + 80;     // [2] accumulator set read out (128 arrivals)
  const uint32_t bar_ready = bar_full + 96;       // S > 1: the other CTAs' stages are free
  const uint32_t bar_recv = bar_full + 104;       // S > 1: the other CTAs' chunks landed here
  const uint32_t bar_end = bar_full + 112;        // every MMA of this CTA finished
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kLinBars + 128);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kLinBars + 136);
  const uint32_t acc_cols = NT <= 128 ? 128u : 256u;  // one sub-tile's accumulator
  const uint32_t tmem_cols = kNbuf * TW * acc_cols;   // <= 512
  const int rank = S == 1 ? 0 : (int)cluster_ctarank();

  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), tmem_cols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&wmap);
    prefetch_tensormap(&xmap);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(bar_full + 8 * i, 1);
      mbar_init(bar_empty + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_acc + 8 * i, 1);
      mbar_init(bar_accfree + 8 * i, 128);
    }
    mbar_init(bar_ready, S > 1 ? S - 1 : 1);
    mbar_init(bar_recv, S > 1 ? (S - 1) * 128 : 1);
    mbar_init(bar_end, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  if (S > 1) cluster_sync_all();  // every CTA's barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // this CTA's tiles and K range
  const int tile0 = S == 1 ? (int)blockIdx.x : (int)blockIdx.x / S;
  const int tstep = S == 1 ? (int)gridDim.x : n_tiles;
  const int kb0 = S == 1 ? 0 : rank * KB / S, kb1 = S == 1 ? KB : (rank + 1) * KB / S;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint32_t bytes = TW * kLinW + (uint32_t)NT * 128;
      const int kper = kb1 - kb0;
      const int n_mine = tile0 < n_tiles ? ((n_tiles - 1 - tile0) / tstep + 1) * kper : 0;
      auto load_w = [&](uint32_t dst, int t, int kb, uint32_t bar) {
#pragma unroll
        for (int w = 0; w < TW; ++w)
          tma_load_2d(dst + w * kLinW, &wmap, kb * 64, (t * TW + w) * 128, bar);
      };
      // The weights do not depend on the previous kernel: the first stages'
      // weight tiles are requested before the programmatic-launch wait, the
      // activation tiles after it.
      const int pre = n_mine < kStages ? n_mine : kStages;
      for (int j = 0; j < pre; ++j) {
        mbar_arrive_expect_tx(bar_full + 8 * j, bytes);
        load_w(sb + j * kStage, tile0 + (j / kper) * tstep, kb0 + j % kper, bar_full + 8 * j);
      }
      griddep_wait();
      for (int j = 0; j < pre; ++j)
        tma_load_2d(sb + j * kStage + TW * kLinW, &xmap, (kb0 + j % kper) * 64, 0,
                    bar_full + 8 * j);
      uint32_t it = (uint32_t)pre;
      bool ok = true;
      for (int j = pre; ok && j < n_mine; ++j, ++it) {
        const int t = tile0 + (j / kper) * tstep, kb = kb0 + j % kper;
        const uint32_t st = it % kStages, round = it / kStages;
        if (*abort_flag || !mbar_wait_bounded(bar_empty + 8 * st, (round & 1) ^ 1)) {
          ok = false;
          break;
        }
        const uint32_t dst = sb + st * kStage;
        mbar_arrive_expect_tx(bar_full + 8 * st, bytes);
        load_w(dst, t, kb, bar_full + 8 * st);
        tma_load_2d(dst + TW * kLinW, &xmap, kb * 64, 0, bar_full + 8 * st);
      }
      if (!ok) {
        *abort_flag = 1;
        set_error(kErrTimeout);
      }
      // copies still in flight land before the CTA moves on
      for (uint32_t j = it > (uint32_t)kStages ? it - kStages : 0; j < it; ++j)
        mbar_wait_bounded(bar_full + 8 * (j % kStages), (j / kStages) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: the whole warp runs the loop (operands
    // warp-uniform), one elected lane issues each MMA and commit ----------------
    griddep_wait();  // the bounded waits below start once the previous kernel is done
    {
      const uint32_t idesc = idesc_f16_f32(kBf16, 128, NT, false, false);
      uint32_t it = 0;
      int i = 0;
      bool ok = true;
      // one answer for the warp, which takes every branch together
      auto wait = [&](uint32_t bar, uint32_t par) {
        return __all_sync(0xffffffffu, !*abort_flag && mbar_wait_bounded(bar, par));
      };
      for (int t = tile0; ok && t < n_tiles; t += tstep, ++i) {
        const int buf = i % kNbuf, use = i / kNbuf;
        if (use > 0 && !wait(bar_accfree + 8 * buf, (use & 1) ^ 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * TW * acc_cols;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const uint32_t st = it % kStages, round = it / kStages;
          if (!wait(bar_full + 8 * st, round & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = sb + st * kStage, b = a + TW * kLinW;
          const bool leader = elect_one();
#pragma unroll
          for (int w = 0; w < TW; ++w)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = smem_desc_sw128(a + w * kLinW + kk * 32, 16, 1024);
              const uint64_t bd = smem_desc_sw128(b + kk * 32, 16, 1024);
              if (leader)
                tc_mma_f16_ss(d + w * acc_cols, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
            }
          if (leader) tc_commit(bar_empty + 8 * st);  // the stage may be refilled
        }
        if (!ok) break;
        if (elect_one()) tc_commit(bar_acc + 8 * buf);
      }
      if (!ok && lane == 0) {
        *abort_flag = 1;
        set_error(kErrTimeout);
      }
      if (elect_one()) tc_commit(bar_end);
      mbar_wait_bounded(bar_end, 0);
    }
  } else {
    // ---------------- epilogue ----------------
    griddep_wait();
    const int q = warp & 3;
    const int nl = q * 32 + lane;  // this thread's output feature within a sub-tile
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const int nchunks = NT / 32;
    auto store_chunk = [&](int n, int c, const float (&v)[32]) {
      if (n >= N) return;
      const float b = bias ? Dt<T>::to_f(bias[n]) : 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int m = c * 32 + j;
        if (m < M) y[(int64_t)m * ldy + n] = Dt<T>::from_f(v[j] + b);
      }
    };
    if constexpr (S == 1) {
      int i = 0;
      for (int t = tile0; t < n_tiles; t += tstep, ++i) {
        const int buf = i % kNbuf, use = i / kNbuf;
        // warp-uniform decision: the TMEM loads below are .sync.aligned
        const bool bad = !mbar_wait_bounded(bar_acc + 8 * buf, use & 1) || *abort_flag;
        if (__any_sync(0xffffffffu, bad)) {
          *abort_flag = 1;
          if (lane == 0) set_error(kErrTimeout);
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int w = 0; w < TW; ++w) {
          const int n = (t * TW + w) * 128 + nl;
          const uint32_t base = tmem + (buf * TW + w) * acc_cols + lane_off;
          for (int c = 0; c < nchunks; ++c) {
            uint32_t r[32];
            tmem_ld32_nowait(base + c * 32, r);
            tmem_wait_ld();
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
            if (w + 1 == TW && c + 1 == nchunks) {
              tc_fence_before();
              mbar_arrive(bar_accfree + 8 * buf);  // the MMA warp may reuse the set
            }
            store_chunk(n, c, v);
          }
        }
      }
    } else {
      const int nlc = (nchunks + S - 1) / S;  // chunks owned per CTA (at most)
      const int t = tile0;
      // every decision below is warp-uniform (.sync.aligned TMEM loads)
      bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar_acc, 0) && !*abort_flag);
      tc_fence_after();
      // this CTA's MMAs are done: its stages may take the other CTAs' chunks
      if (ok && threadIdx.x == 64) {
        for (int o = 0; o < S; ++o)
          if (o != rank) mbar_arrive_remote(mapa_shared(bar_ready, (uint32_t)o));
      }
      ok = __all_sync(0xffffffffu, ok && mbar_wait_cluster_bounded(bar_ready, 0));
      if (ok) {
        for (int c = 0; c < nchunks; ++c) {
          const int o = c % S;
          if (o == rank) continue;
          uint32_t r[32];
          tmem_ld32_nowait(tmem + lane_off + c * 32, r);
          tmem_wait_ld();
          const uint32_t dst =
              mapa_shared(sb + (uint32_t)((rank * nlc + c / S) * kLinChunk + nl * 16), (uint32_t)o);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4)
            st_cluster_v4(dst + j4 * 128 * 16, __uint_as_float(r[4 * j4]),
                          __uint_as_float(r[4 * j4 + 1]), __uint_as_float(r[4 * j4 + 2]),
                          __uint_as_float(r[4 * j4 + 3]));
        }
        for (int o = 0; o < S; ++o)
          if (o != rank) mbar_arrive_remote(mapa_shared(bar_recv, (uint32_t)o));
        ok = __all_sync(0xffffffffu, mbar_wait_cluster_bounded(bar_recv, 0));
      }
      if (ok) {
        const int n = t * 128 + nl;
        for (int c = rank; c < nchunks; c += S) {
          uint32_t r[32];
          tmem_ld32_nowait(tmem + lane_off + c * 32, r);
          tmem_wait_ld();
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          for (int s = 0; s < S; ++s) {  // own partial, then the others' in rank order
            if (s == rank) continue;
            const float4* src = reinterpret_cast<const float4*>(
                smem + (size_t)(s * nlc + c / S) * kLinChunk + nl * 16);
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 p = src[j4 * 128];
              v[4 * j4] += p.x;
              v[4 * j4 + 1] += p.y;
              v[4 * j4 + 2] += p.z;
              v[4 * j4 + 3] += p.w;
            }
          }
          store_chunk(n, c, v);
        }
      } else {
        *abort_flag = 1;
        if (lane == 0) set_error(kErrTimeout);
      }
    }
  }
  // programmatic launch: the next kernel may be scheduled now; it waits for
  // this grid's completion before reading anything
  griddep_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (S > 1) cluster_sync_all();  // no CTA leaves while another may still write to it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

}  // namespace nb

namespace nbh {

// Shape of the launch: TW (128-row weight sub-tiles per tile) and S (CTAs
// per cluster splitting K).  Default: 256-row tiles (TW = 2) on persistent
// CTAs, the most weight bytes in flight per SM.  NB_LINEAR_SPLIT=2..4 takes
// the cluster split-K path with 128-row tiles, NB_LINEAR_SPLIT=1 128-row
// tiles without a split (diagnostics and tests).
struct LinPlan {
  int tw, s;
};
inline LinPlan linear_plan(int KB) {
  const char* e = getenv("NB_LINEAR_SPLIT");
  if (e && e[0] >= '1' && e[0] <= '4') return LinPlan{1, std::min(e[0] - '0', std::max(1, KB))};
  return LinPlan{2, 1};
}

template <typename T, int S, int TW>
int launch_linear_s(const CUtensorMap& wm, const CUtensorMap& xm, void* y, int64_t ldy,
                    const void* bias, int M, int N, int NT, int KB, cudaStream_t st) {
  auto kern = nb::linear_tc_kernel<T, S, TW>;
  if (int r = ensure_max_smem((const void*)kern, nb::kLinSmem, "linear_tc")) return r;
  const int n_tiles = (N + 128 * TW - 1) / (128 * TW);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  cfg.blockDim = dim3(nb::kLinThreads);
  cfg.dynamicSmemBytes = nb::kLinSmem;
  cfg.stream = st;
  cfg.gridDim = dim3(S == 1 ? (unsigned)std::min(n_tiles, num_sms()) : (unsigned)(n_tiles * S));
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  if (pdl_enabled()) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
    ++cfg.numAttrs;
  }
  if (S > 1) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
    attr[cfg.numAttrs].val.clusterDim.x = S;
    attr[cfg.numAttrs].val.clusterDim.y = 1;
    attr[cfg.numAttrs].val.clusterDim.z = 1;
    ++cfg.numAttrs;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, wm, xm, (T*)y, ldy, (const T*)bias, M, N, NT,
                                     n_tiles, KB);
  if (e != cudaSuccess) return fail(NB_ERR_CUDA, "linear_tc launch: %s", cudaGetErrorString(e));
  return check_launch("linear_tc");
}

template <typename T>
int launch_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, const void* bias,
                  void* y, int64_t ldy, int M, int N, int K, int dtype, cudaStream_t st) {
  const int NT = (M + 31) / 32 * 32;
  const int KB = (K + 63) / 64;
  CUtensorMap wm, xm;
  int rc = tensor_map_2d(&wm, w, dtype, (uint64_t)K, (uint64_t)N, (uint64_t)ldw * 2, 64, 128);
  if (!rc) rc = tensor_map_2d(&xm, x, dtype, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 2, 64, NT);
  if (rc) return rc;
  const LinPlan p = linear_plan(KB);
  if (p.tw == 2) return launch_linear_s<T, 1, 2>(wm, xm, y, ldy, bias, M, N, NT, KB, st);
  switch (p.s) {
    case 2: return launch_linear_s<T, 2, 1>(wm, xm, y, ldy, bias, M, N, NT, KB, st);
    case 3: return launch_linear_s<T, 3, 1>(wm, xm, y, ldy, bias, M, N, NT, KB, st);
    case 4: return launch_linear_s<T, 4, 1>(wm, xm, y, ldy, bias, M, N, NT, KB, st);
    default: return launch_linear_s<T, 1, 1>(wm, xm, y, ldy, bias, M, N, NT, KB, st);
  }
}

}  // namespace nbh

extern "C" {

int nb_linear(const void* x, int64_t x_stride, const void* weight, int64_t w_stride,
              const void* bias, void* y, int64_t y_stride, int M, int N, int K, int dtype,
              void* stream) {
  using namespace nbh;
  if (dtype != NB_DTYPE_BF16 && dtype != NB_DTYPE_F16)
    return fail(NB_ERR_UNSUPPORTED, "nb_linear takes bf16 or fp16");
  if (!x || !weight || !y) return fail(NB_ERR_INVALID_ARG, "null pointer");
  if (M < 0 || N <= 0 || K <= 0) return fail(NB_ERR_INVALID_ARG, "bad sizes");
  if (M == 0) return NB_OK;
  if (M > 256) return fail(NB_ERR_UNSUPPORTED, "nb_linear is for at most 256 rows (got %d)", M);
  if (x_stride < K || w_stride < K || y_stride < N)
    return fail(NB_ERR_INVALID_ARG, "row stride too small");
  if (K % 8 || x_stride % 8 || w_stride % 8 || ((uintptr_t)x & 15) || ((uintptr_t)weight & 15))
    return fail(NB_ERR_UNSUPPORTED, "nb_linear needs 16-byte aligned rows of x and weight");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == NB_DTYPE_BF16)
    return launch_linear<__nv_bfloat16>(x, x_stride, weight, w_stride, bias, y, y_stride, M, N, K,
                                        dtype, st);
  return launch_linear<__half>(x, x_stride, weight, w_stride, bias, y, y_stride, M, N, K, dtype,
                               st);
}

}  // extern "C"
