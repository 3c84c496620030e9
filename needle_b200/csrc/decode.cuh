// Paged split-K decode attention and its merge kernel.
//
// Tensor-core path (bf16/fp16, block_size 16, head_dim 64/128, any group):
//   * one CTA of WARPS warps per (split, kv head, chunk of <= 8 query heads of
//     its group, sequence); a split is a run of
//     `pps` consecutive pages (KV blocks) of the sequence;
//   * warp w owns pages w, w+WARPS, ... of its split and runs its own
//     STAGES-deep TMA pipeline: each 16-token page of K and of V lands in a
//     private shared-memory slot (128-byte swizzled, 2 KB per 64 columns),
//     signalled by a per-slot mbarrier.  Warps never wait on each other
//     until the final in-CTA merge;
//   * per page, S^T[16 tok x 8 heads] = K_page . Q^T on mma.m16n8k16 (the
//     group's <= 8 query heads are the N dimension, so K is read from shared
//     memory once for all of them), an online softmax with warp shuffles
//     across the 8 lanes that share a head, P^T re-laid out in registers
//     with movmatrix, and O^T[D x 8] += V_page^T . P^T on mma again;
//   * the warps' (m, l, O) are merged through shared memory; a sequence
//     with one split writes the output directly, otherwise fp32 partials go
//     to the workspace and decode_merge_kernel combines them.
// SIMT path (fp32, or shapes the tensor-core path does not take): the same
// split/merge structure with one token per warp step and shuffle-reduced
// dot products; used for the fp32 configurations where exactness matters
// more than speed.
//
// Softmax runs in base 2: scores are multiplied by scale * log2(e) and
// exponentiated with exp2f, so m (the running max) is in log2 units in the
// partials too.
#pragma once
#include "nb_common.cuh"

namespace nb {

constexpr float kLog2e = 1.4426950408889634f;

template <int D> struct TcGeom {
  static constexpr int kHalves = D / 64;                 // 64-column (128-byte) slabs per row
  static constexpr int kSlabBytes = 16 * 128;            // 16 rows x 128 B
  static constexpr int kPageBytes = kHalves * kSlabBytes;  // one page of K (or V)
  static constexpr int kStageBytes = 2 * kPageBytes;       // K + V
};

// Shared-memory address of 16-byte chunk c (of D/8) in row r of a page laid
// out by TMA with 128-byte swizzle: slab c/8, chunk (c%8) XOR (r%8).
__device__ __forceinline__ uint32_t swz_addr(uint32_t page, int r, int c) {
  return page + ((c >> 3) << 11) + (r << 7) + ((((c & 7) ^ (r & 7))) << 4);
}

__device__ __forceinline__ void decode_extent(int ctx, int maxb, int bs, int pps, int& n_tok,
                                              int& n_pages, int& n_splits) {
  // needle attends over context_lens + 1 tokens and reads at most the
  // table's maxb pages (attention.py:297-301).
  int t = ctx + 1;
  if (t > maxb * bs) t = maxb * bs;
  if (t < 0) t = 0;
  n_tok = t;
  n_pages = (t + bs - 1) / bs;
  n_splits = (n_pages + pps - 1) / pps;
  if (n_splits < 1) n_splits = 1;
}

// NH: 8-head MMA column tiles per CTA (1: up to 8 query heads of a KV head;
// 2: up to 16, for groups above 8, so each page is read by one CTA).
template <typename T, int D, int WARPS, int STAGES, int NH>
__global__ void __launch_bounds__(WARPS * 32)
    paged_decode_tc_kernel(const __grid_constant__ CUtensorMap kv_map, const T* __restrict__ q,
                           int64_t q_sb, int64_t q_sh, const int32_t* __restrict__ bt,
                           int64_t bt_stride, int maxb, const int32_t* __restrict__ ctx_lens,
                           int kvh, int group, int num_blocks, float scale_log2, int pps,
                           T* __restrict__ out, int64_t o_sb, int64_t o_sh,
                           float* __restrict__ part_o, float2* __restrict__ part_ml,
                           int max_splits) {
  using G = TcGeom<D>;
  constexpr int NK = D / 16;
  // Launched with programmatic stream serialisation: everything this grid
  // reads (q, the cache pages, the block table, context lengths) may come
  // from the kernel just before it, so wait for that grid first.
  griddep_wait();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  // grid.y = kv head x chunks of up to 8 NH query heads of its group: groups
  // above 8 NH run as several CTAs that read the same pages (adjacent in the
  // grid, so the second read of a page is usually an L2 hit)
  constexpr int HN = 8 * NH;  // query heads per CTA
  const int nhc = (group + HN - 1) / HN;
  const int split = blockIdx.x, h = blockIdx.y / nhc, b = blockIdx.z;
  const int n0 = (blockIdx.y - h * nhc) * HN;
  const int gcount = min(HN, group - n0);
  const int ctx = __ldg(ctx_lens + b);
  if (ctx < 0 && threadIdx.x == 0 && split == 0 && n0 == 0) set_error(kErrPosition);
  int n_tok, n_pages, n_splits;
  decode_extent(ctx, maxb, 16, pps, n_tok, n_pages, n_splits);
  if (split >= n_splits) return;
  const int p0 = split * pps;
  const int p1 = min(p0 + pps, n_pages);
  const int n_w = max(0, (p1 - p0 - warp + WARPS - 1) / WARPS);

  uint8_t* wbase = smem + warp * STAGES * G::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + WARPS * STAGES * G::kStageBytes) +
                   warp * STAGES;
  const uint32_t wbase_u = smem_u32(wbase);
  const uint32_t bar_u = smem_u32(bars);

  // Block ids of this warp's pages: lane i holds page p0 + warp + WARPS * i.
  int my_row = -16;  // first cache row of the page's K slab (OOB -> zero fill)
  if (lane < n_w) {
    const int phys = __ldg(bt + (int64_t)b * bt_stride + p0 + warp + WARPS * lane);
    if (phys >= 0 && phys < num_blocks) my_row = (phys * kvh + h) * 16;
    else set_error(kErrBlockId);
  }
  const int v_off = num_blocks * kvh * 16;  // V rows follow all K rows

  if (lane == 0) {
    prefetch_tensormap(&kv_map);
    for (int s = 0; s < STAGES; ++s) mbar_init(bar_u + 8 * s, 1);
    fence_mbar_init();
  }
  __syncwarp();

  auto issue = [&](int i, int row) {  // lane 0 only
    const int s = i % STAGES;
    const uint32_t bar = bar_u + 8 * s;
    const uint32_t kdst = wbase_u + s * G::kStageBytes;
    const uint32_t vdst = kdst + G::kPageBytes;
    mbar_arrive_expect_tx(bar, G::kStageBytes);
    const int vrow = row < 0 ? row : row + v_off;
#pragma unroll
    for (int hf = 0; hf < G::kHalves; ++hf) {
      tma_load_2d(kdst + hf * G::kSlabBytes, &kv_map, hf * 64, row, bar);
      tma_load_2d(vdst + hf * G::kSlabBytes, &kv_map, hf * 64, vrow, bar);
    }
  };

#pragma unroll
  for (int i = 0; i < STAGES; ++i) {
    const int row = __shfl_sync(0xffffffffu, my_row, i);
    if (lane == 0 && i < n_w) issue(i, row);
  }

  // Q^T as the B operand (k = d, n = head): in column tile nt, lane holds
  // head 8 nt + g, d pairs 2*t4.
  uint32_t qf[NH][NK][2];
#pragma unroll
  for (int nt = 0; nt < NH; ++nt) {
    const bool hv = 8 * nt + g < gcount;
    const T* qrow =
        q + (int64_t)b * q_sb + (int64_t)(h * group + n0 + (hv ? 8 * nt + g : 0)) * q_sh;
#pragma unroll
    for (int kk = 0; kk < NK; ++kk) {
      qf[nt][kk][0] =
          hv ? __ldg(reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * t4)) : 0u;
      qf[nt][kk][1] =
          hv ? __ldg(reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 8 + 2 * t4)) : 0u;
    }
  }

  float o[NH][NK][4];
  float m0[NH], m1[NH], l0[NH], l1[NH];
#pragma unroll
  for (int nt = 0; nt < NH; ++nt) {
#pragma unroll
    for (int mt = 0; mt < NK; ++mt) o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.f;
    m0[nt] = m1[nt] = -INFINITY;
    l0[nt] = l1[nt] = 0.f;
  }
  const int mi = lane >> 3;
  bool ok = true;
  int consumed = 0;

  for (int i = 0; i < n_w; ++i) {
    const int s = i % STAGES;
    const bool got = mbar_wait_bounded(bar_u + 8 * s, (i / STAGES) & 1);
    if (__any_sync(0xffffffffu, !got)) { ok = false; break; }
    consumed = i + 1;
    const uint32_t kb = wbase_u + s * G::kStageBytes;
    const uint32_t vb = kb + G::kPageBytes;

    // S^T = K . Q^T  (16 tokens x 8 NH heads); the K fragments serve every
    // column tile; two independent accumulation chains per tile halve the
    // MMA dependency depth
    float sc[NH][4], sd[NH][4];
#pragma unroll
    for (int nt = 0; nt < NH; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[nt][e] = sd[nt][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < NK; kk += 2) {
      uint32_t a[4], a2[4];
      ldmatrix_x4(a, swz_addr(kb, (lane & 7) + ((mi & 1) << 3), kk * 2 + (mi >> 1)));
      ldmatrix_x4(a2, swz_addr(kb, (lane & 7) + ((mi & 1) << 3), kk * 2 + 2 + (mi >> 1)));
#pragma unroll
      for (int nt = 0; nt < NH; ++nt) {
        Mma<T>::run(sc[nt], a, qf[nt][kk][0], qf[nt][kk][1]);
        Mma<T>::run(sd[nt], a2, qf[nt][kk + 1][0], qf[nt][kk + 1][1]);
      }
    }
    const int tok = (p0 + warp + WARPS * i) * 16 + g;
    uint32_t pb0[NH], pb1[NH];
#pragma unroll
    for (int nt = 0; nt < NH; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[nt][e] += sd[nt][e];
      const float x0 = tok < n_tok ? sc[nt][0] * scale_log2 : -INFINITY;
      const float x1 = tok < n_tok ? sc[nt][1] * scale_log2 : -INFINITY;
      const float x2 = tok + 8 < n_tok ? sc[nt][2] * scale_log2 : -INFINITY;
      const float x3 = tok + 8 < n_tok ? sc[nt][3] * scale_log2 : -INFINITY;
      float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
      for (int sh = 4; sh < 32; sh <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, sh));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, sh));
      }
      // every page holds at least one valid token, so mx is finite
      const float mn0 = fmaxf(m0[nt], mx0), mn1 = fmaxf(m1[nt], mx1);
      const float al0 = exp2f(m0[nt] - mn0), al1 = exp2f(m1[nt] - mn1);
      const float e0 = exp2f(x0 - mn0), e1 = exp2f(x1 - mn1);
      const float e2 = exp2f(x2 - mn0), e3 = exp2f(x3 - mn1);
      l0[nt] = l0[nt] * al0 + (e0 + e2);
      l1[nt] = l1[nt] * al1 + (e1 + e3);
      m0[nt] = mn0;
      m1[nt] = mn1;
#pragma unroll
      for (int mt = 0; mt < NK; ++mt) {
        o[nt][mt][0] *= al0; o[nt][mt][1] *= al1; o[nt][mt][2] *= al0; o[nt][mt][3] *= al1;
      }
      // P^T as the B operand (k = token, n = head)
      pb0[nt] = movmatrix_trans(Mma<T>::pack(e0, e1));
      pb1[nt] = movmatrix_trans(Mma<T>::pack(e2, e3));
    }
    // O^T += V^T . P^T   (D x 8 NH); the V fragments serve every column tile
#pragma unroll
    for (int mt = 0; mt < NK; ++mt) {
      uint32_t a[4];
      ldmatrix_x4_trans(a, swz_addr(vb, (lane & 7) + ((mi >> 1) << 3), mt * 2 + (mi & 1)));
#pragma unroll
      for (int nt = 0; nt < NH; ++nt) Mma<T>::run(o[nt][mt], a, pb0[nt], pb1[nt]);
    }
    __syncwarp();
    const int nxt = i + STAGES;
    const int row = __shfl_sync(0xffffffffu, my_row, nxt & 31);
    if (lane == 0 && nxt < n_w) {
      fence_proxy_async_smem();
      issue(nxt, row);
    }
  }
  if (!ok) {
    if (lane == 0) {
      set_error(kErrTimeout);
      // let the copies still in flight land before the slots are reused
      for (int i = consumed; i < min(n_w, consumed + STAGES); ++i)
        mbar_wait_bounded(bar_u + 8 * (i % STAGES), (i / STAGES) & 1);
    }
    __syncwarp();
  }

#pragma unroll
  for (int nt = 0; nt < NH; ++nt)
#pragma unroll
    for (int sh = 4; sh < 32; sh <<= 1) {
      l0[nt] += __shfl_xor_sync(0xffffffffu, l0[nt], sh);
      l1[nt] += __shfl_xor_sync(0xffffffffu, l1[nt], sh);
    }

  // Let the merge kernel (launched with programmatic stream serialisation)
  // get scheduled while this grid drains; it waits for our completion before
  // reading any partial.
  griddep_launch_dependents();

  // In-CTA merge of the warps through shared memory (pipeline slots reused).
  __syncthreads();
  float* sm_o = reinterpret_cast<float*>(smem);            // [warps][HN][D]
  float* sm_m = sm_o + WARPS * HN * D;                   // [warps][HN]
  float* sm_l = sm_m + WARPS * HN;
#pragma unroll
  for (int nt = 0; nt < NH; ++nt) {
    const int r0 = warp * HN + 8 * nt + 2 * t4;  // heads 8 nt + 2 t4, + 1
#pragma unroll
    for (int mt = 0; mt < NK; ++mt) {
      const int d = mt * 16 + g;
      sm_o[r0 * D + d] = o[nt][mt][0];
      sm_o[(r0 + 1) * D + d] = o[nt][mt][1];
      sm_o[r0 * D + d + 8] = o[nt][mt][2];
      sm_o[(r0 + 1) * D + d + 8] = o[nt][mt][3];
    }
    if (g == 0) {
      sm_m[r0] = m0[nt];
      sm_m[r0 + 1] = m1[nt];
      sm_l[r0] = l0[nt];
      sm_l[r0 + 1] = l1[nt];
    }
  }
  __syncthreads();
  const int H = kvh * group;
  for (int idx = threadIdx.x; idx < gcount * D; idx += WARPS * 32) {
    const int n = idx / D, d = idx - n * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, sm_m[w * HN + n]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      const float mw = sm_m[w * HN + n];
      const float e = mw == -INFINITY ? 0.f : exp2f(mw - M);
      L += sm_l[w * HN + n] * e;
      O += sm_o[(w * HN + n) * D + d] * e;
    }
    const int qh = h * group + n0 + n;
    if (n_splits == 1) {
      out[(int64_t)b * o_sb + (int64_t)qh * o_sh + d] = Dt<T>::from_f(L > 0.f ? O / L : 0.f);
    } else {
      const int64_t pi = ((int64_t)b * H + qh) * max_splits + split;
      part_o[pi * D + d] = O;
      if (d == 0) part_ml[pi] = make_float2(M, L);
    }
  }
}

// SIMT split-K decode: any block size, head_dim % 32 == 0 (<= 256), any
// group (heads beyond GMAX go to further CTAs along grid.y).
template <typename T, int D, int GMAX>
__global__ void __launch_bounds__(128)
    paged_decode_simt_kernel(const T* __restrict__ cache, int num_blocks, int kvh, int bs,
                             const T* __restrict__ q, int64_t q_sb, int64_t q_sh,
                             const int32_t* __restrict__ bt, int64_t bt_stride, int maxb,
                             const int32_t* __restrict__ ctx_lens, int group, float scale_log2,
                             int pps, T* __restrict__ out, int64_t o_sb, int64_t o_sh,
                             float* __restrict__ part_o, float2* __restrict__ part_ml,
                             int max_splits) {
  constexpr int EPL = D / 32;
  griddep_wait();  // see paged_decode_tc_kernel
  extern __shared__ float sm_f[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nhc = (group + GMAX - 1) / GMAX;
  const int h = blockIdx.y / nhc, hc = blockIdx.y - h * nhc;
  const int split = blockIdx.x, b = blockIdx.z;
  const int n0 = hc * GMAX;
  const int gcount = min(GMAX, group - n0);
  const int ctx = __ldg(ctx_lens + b);
  if (ctx < 0 && threadIdx.x == 0 && split == 0 && hc == 0) set_error(kErrPosition);
  int n_tok, n_pages, n_splits;
  decode_extent(ctx, maxb, bs, pps, n_tok, n_pages, n_splits);
  if (split >= n_splits) return;
  const int t_begin = split * pps * bs;
  const int t_end = min(t_begin + pps * bs, n_tok);

  float qv[GMAX][EPL], acc[GMAX][EPL], m[GMAX], l[GMAX];
#pragma unroll
  for (int n = 0; n < GMAX; ++n) {
    m[n] = -INFINITY;
    l[n] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      acc[n][e] = 0.f;
      qv[n][e] = n < gcount ? Dt<T>::to_f(q[(int64_t)b * q_sb +
                                            (int64_t)(h * group + n0 + n) * q_sh + lane * EPL + e])
                            : 0.f;
    }
  }
  const int64_t vbase = (int64_t)num_blocks * kvh * bs * D;
  for (int tk = t_begin + warp; tk < t_end; tk += 4) {
    const int page = tk / bs, off = tk - page * bs;
    const int phys = __ldg(bt + (int64_t)b * bt_stride + page);
    if (phys < 0 || phys >= num_blocks) {
      if (lane == 0) set_error(kErrBlockId);
      continue;
    }
    const int64_t row = (((int64_t)phys * kvh + h) * bs + off) * D + lane * EPL;
    float kx[EPL], vx[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      kx[e] = Dt<T>::to_f(cache[row + e]);
      vx[e] = Dt<T>::to_f(cache[vbase + row + e]);
    }
#pragma unroll
    for (int n = 0; n < GMAX; ++n) {
      if (n >= gcount) break;
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) s = fmaf(qv[n][e], kx[e], s);
      s = warp_sum(s) * scale_log2;
      const float mn = fmaxf(m[n], s);
      const float al = exp2f(m[n] - mn);
      const float p = exp2f(s - mn);
      l[n] = l[n] * al + p;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[n][e] = fmaf(acc[n][e], al, p * vx[e]);
      m[n] = mn;
    }
  }
  // merge the 4 warps
  float* sm_o = sm_f;                      // [4][GMAX][D]
  float* sm_m = sm_o + 4 * GMAX * D;       // [4][GMAX]
  float* sm_l = sm_m + 4 * GMAX;
#pragma unroll
  for (int n = 0; n < GMAX; ++n) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) sm_o[(warp * GMAX + n) * D + lane * EPL + e] = acc[n][e];
    if (lane == 0) {
      sm_m[warp * GMAX + n] = m[n];
      sm_l[warp * GMAX + n] = l[n];
    }
  }
  __syncthreads();
  const int H = kvh * group;
  for (int idx = threadIdx.x; idx < gcount * D; idx += 128) {
    const int n = idx / D, d = idx - n * D;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w * GMAX + n]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float mw = sm_m[w * GMAX + n];
      const float e = mw == -INFINITY ? 0.f : exp2f(mw - M);
      L += sm_l[w * GMAX + n] * e;
      O += sm_o[(w * GMAX + n) * D + d] * e;
    }
    const int qh = h * group + n0 + n;
    if (n_splits == 1) {
      out[(int64_t)b * o_sb + (int64_t)qh * o_sh + d] = Dt<T>::from_f(L > 0.f ? O / L : 0.f);
    } else {
      const int64_t pi = ((int64_t)b * H + qh) * max_splits + split;
      part_o[pi * D + d] = O;
      if (d == 0) part_ml[pi] = make_float2(M, L);
    }
  }
}

// Combine the split partials of every (sequence, query head) that has more
// than one split.  One warp per (sequence, head): lane s reads split s's
// (m, l), the warp reduces max and normaliser with shuffles, then every lane
// accumulates its D/32 columns over the splits (independent loads, one
// memory round trip).  Launched with programmatic stream serialisation: the
// griddepcontrol.wait below returns once the split kernel has completed and
// its partials are visible.
template <typename T>
__global__ void __launch_bounds__(128)
    decode_merge_kernel(const float* __restrict__ part_o, const float2* __restrict__ part_ml,
                        const int32_t* __restrict__ ctx_lens, int maxb, int bs, int pps, int B,
                        int H, int D, int max_splits, T* __restrict__ out, int64_t o_sb,
                        int64_t o_sh) {
  griddep_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = blockIdx.x * 4 + warp;
  if (pair >= B * H) return;
  const int b = pair / H, qh = pair - b * H;
  int n_tok, n_pages, n_splits;
  decode_extent(__ldg(ctx_lens + b), maxb, bs, pps, n_tok, n_pages, n_splits);
  if (n_splits <= 1) return;
  const int64_t base = (int64_t)pair * max_splits;
  float M = -INFINITY;
  for (int s0 = 0; s0 < n_splits; s0 += 32) {
    const int s = s0 + lane;
    if (s < n_splits) M = fmaxf(M, part_ml[base + s].x);
  }
  M = warp_max(M);
  float L = 0.f;
  for (int s0 = 0; s0 < n_splits; s0 += 32) {
    const int s = s0 + lane;
    if (s < n_splits) {
      const float2 ml = part_ml[base + s];
      L += ml.y * (ml.x == -INFINITY ? 0.f : exp2f(ml.x - M));
    }
  }
  L = warp_sum(L);
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const int epl = D / 32;  // columns per lane (D is a multiple of 32)
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  for (int s0 = 0; s0 < n_splits; s0 += 32) {
    const int sl = s0 + lane;
    const float2 ml = sl < n_splits ? part_ml[base + sl] : make_float2(-INFINITY, 0.f);
    const float wl = ml.x == -INFINITY ? 0.f : exp2f(ml.x - M);
    const int cnt = min(32, n_splits - s0);
    // four splits per step with their loads issued together (one round trip)
    for (int j = 0; j < cnt; j += 4) {
      float w[4], x[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int jj = min(j + u, cnt - 1);
        w[u] = __shfl_sync(0xffffffffu, wl, jj);
        if (j + u >= cnt) w[u] = 0.f;
        const float* src = part_o + (base + s0 + jj) * D + lane * epl;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < epl) x[u][e] = __ldg(src + e);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < epl) acc[e] = fmaf(x[u][e], w[u], acc[e]);
    }
  }
  T* dst = out + (int64_t)b * o_sb + (int64_t)qh * o_sh + lane * epl;
#pragma unroll
  for (int e = 0; e < 8; ++e)
    if (e < epl) dst[e] = Dt<T>::from_f(acc[e] * inv);
}

}  // namespace nb

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
namespace nbh {

// Tensor-core decode configuration: warps per CTA and TMA pipeline depth per
// warp.  Each warp keeps one page id per lane, so a split holds at most
// 32 * warps pages.
struct TcCfg {
  int warps, stages;
};

inline TcCfg decode_cfg() {
  static TcCfg cfg = [] {
    TcCfg c{4, 2};
    if (const char* e = getenv("NB_DECODE_CFG")) {  // tuning knob: "warps,stages"
      int w = 0, s = 0;
      if (sscanf(e, "%d,%d", &w, &s) == 2 &&
          ((w == 4 && (s == 2 || s == 3 || s == 4)) || (w == 8 && s == 2)))
        c = TcCfg{w, s};
    }
    return c;
  }();
  return cfg;
}

inline bool decode_n16_enabled() {
  static int on = [] {
    const char* e = getenv("NB_DECODE_N16");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return on != 0;
}

template <typename T, int D, int WARPS, int STAGES>
int launch_decode_tc(const CUtensorMap& map, const void* q, int64_t qsb, int64_t qsh,
                     const int32_t* bt, int64_t bts, int maxb, const int32_t* ctx, int kvh,
                     int group, int nblk, float scale_log2, int pps, void* out, int64_t osb,
                     int64_t osh, float* po, float2* pml, int max_splits, int B, cudaStream_t st) {
  using G = nb::TcGeom<D>;
  const size_t smem =
      1024 + (size_t)WARPS * STAGES * G::kStageBytes + (size_t)WARPS * STAGES * 8;
  // groups above 8: 16 heads per CTA (two MMA column tiles), so a page is
  // read by one CTA (NB_DECODE_N16=0 keeps 8-head chunks; diagnostics)
  const bool n16 = group > 8 && decode_n16_enabled();
  auto kern = n16 ? nb::paged_decode_tc_kernel<T, D, WARPS, STAGES, 2>
                  : nb::paged_decode_tc_kernel<T, D, WARPS, STAGES, 1>;
  if (int rc = ensure_max_smem((const void*)kern, (int)smem, "paged_decode_tc")) return rc;
  const int hn = n16 ? 16 : 8;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  pdl_config(cfg, attr, dim3(max_splits, kvh * ((group + hn - 1) / hn), B), dim3(WARPS * 32),
             smem, st);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, map, (const T*)q, qsb, qsh, bt, bts, maxb,
                                           ctx, kvh, group, nblk, scale_log2, pps, (T*)out, osb,
                                           osh, po, pml, max_splits);
  if (e != cudaSuccess) return fail(NB_ERR_CUDA, "paged_decode_tc launch: %s", cudaGetErrorString(e));
  return check_launch("paged_decode_tc");
}

template <typename T, int D>
int dispatch_decode_tc(const CUtensorMap& map, const void* q, int64_t qsb, int64_t qsh,
                       const int32_t* bt, int64_t bts, int maxb, const int32_t* ctx, int kvh,
                       int group, int nblk, float sl2, int pps, void* out, int64_t osb,
                       int64_t osh, float* po, float2* pml, int ms, int B, cudaStream_t st) {
  const TcCfg c = decode_cfg();
#define NB_TC(W, S)                                                                           \
  if (c.warps == W && c.stages == S)                                                          \
    return launch_decode_tc<T, D, W, S>(map, q, qsb, qsh, bt, bts, maxb, ctx, kvh, group,     \
                                        nblk, sl2, pps, out, osb, osh, po, pml, ms, B, st);
  NB_TC(4, 3)
  NB_TC(4, 4)
  NB_TC(8, 2)
#undef NB_TC
  return launch_decode_tc<T, D, 4, 2>(map, q, qsb, qsh, bt, bts, maxb, ctx, kvh, group, nblk, sl2,
                                      pps, out, osb, osh, po, pml, ms, B, st);
}

template <typename T, int D>
int launch_decode_simt(const void* cache, int nblk, int kvh, int bs, const void* q, int64_t qsb,
                       int64_t qsh, const int32_t* bt, int64_t bts, int maxb, const int32_t* ctx,
                       int group, float scale_log2, int pps, void* out, int64_t osb, int64_t osh,
                       float* po, float2* pml, int max_splits, int B, cudaStream_t st) {
  constexpr int GMAX = 8;
  const size_t smem = sizeof(float) * (4 * GMAX * D + 8 * GMAX);
  auto kern = nb::paged_decode_simt_kernel<T, D, GMAX>;
  if (int rc = ensure_max_smem((const void*)kern, (int)smem, "paged_decode_simt")) return rc;
  const int nhc = (group + GMAX - 1) / GMAX;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  pdl_config(cfg, attr, dim3(max_splits, kvh * nhc, B), dim3(128), smem, st);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, (const T*)cache, nblk, kvh, bs, (const T*)q,
                                           qsb, qsh, bt, bts, maxb, ctx, group, scale_log2, pps,
                                           (T*)out, osb, osh, po, pml, max_splits);
  if (e != cudaSuccess)
    return fail(NB_ERR_CUDA, "paged_decode_simt launch: %s", cudaGetErrorString(e));
  return check_launch("paged_decode_simt");
}

template <typename T>
int launch_decode_simt_d(int D, const void* cache, int nblk, int kvh, int bs, const void* q,
                         int64_t qsb, int64_t qsh, const int32_t* bt, int64_t bts, int maxb,
                         const int32_t* ctx, int group, float sl2, int pps, void* out,
                         int64_t osb, int64_t osh, float* po, float2* pml, int ms, int B,
                         cudaStream_t st) {
  switch (D) {
    case 32: return launch_decode_simt<T, 32>(cache, nblk, kvh, bs, q, qsb, qsh, bt, bts, maxb, ctx, group, sl2, pps, out, osb, osh, po, pml, ms, B, st);
    case 64: return launch_decode_simt<T, 64>(cache, nblk, kvh, bs, q, qsb, qsh, bt, bts, maxb, ctx, group, sl2, pps, out, osb, osh, po, pml, ms, B, st);
    case 96: return launch_decode_simt<T, 96>(cache, nblk, kvh, bs, q, qsb, qsh, bt, bts, maxb, ctx, group, sl2, pps, out, osb, osh, po, pml, ms, B, st);
    case 128: return launch_decode_simt<T, 128>(cache, nblk, kvh, bs, q, qsb, qsh, bt, bts, maxb, ctx, group, sl2, pps, out, osb, osh, po, pml, ms, B, st);
    case 256: return launch_decode_simt<T, 256>(cache, nblk, kvh, bs, q, qsb, qsh, bt, bts, maxb, ctx, group, sl2, pps, out, osb, osh, po, pml, ms, B, st);
    default: return fail(NB_ERR_UNSUPPORTED, "head_dim %d not supported by paged decode", D);
  }
}

template <typename T>
int launch_merge(const float* po, const float2* pml, const int32_t* ctx, int maxb, int bs, int pps,
                 int B, int H, int D, int max_splits, void* out, int64_t osb, int64_t osh,
                 cudaStream_t st) {
  const int pairs = B * H;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  pdl_config(cfg, attr, dim3((pairs + 3) / 4), dim3(128), 0, st);
  cudaError_t e = cudaLaunchKernelEx(&cfg, nb::decode_merge_kernel<T>, po, pml, ctx, maxb, bs,
                                     pps, B, H, D, max_splits, (T*)out, osb, osh);
  if (e != cudaSuccess) return fail(NB_ERR_CUDA, "decode_merge launch: %s", cudaGetErrorString(e));
  return check_launch("decode_merge");
}

inline int max_pages_per_split_tc() { return 32 * decode_cfg().warps; }

}  // namespace nbh

extern "C" {

int nb_paged_decode_plan(int num_seqs, int num_kv_heads, int max_blocks_per_seq, int block_size,
                         int* pages_per_split, int* max_splits) {
  using namespace nbh;
  if (!pages_per_split || !max_splits) return fail(NB_ERR_INVALID_ARG, "null output pointer");
  if (num_seqs <= 0 || num_kv_heads <= 0 || max_blocks_per_seq <= 0 || block_size <= 0)
    return fail(NB_ERR_INVALID_ARG, "non-positive shape");
  // Splits exist only to give the GPU enough CTAs: aim for about four waves
  // of the three 4-warp CTAs that fit on an SM (66 KB of shared memory each).
  // When sequences x KV heads already reach that, every sequence is one
  // split (no partials, no merge).  Otherwise the longest sequence (the
  // block-table width) is cut into that many splits.  At config 2 (64 x 8
  // heads, up to 256 pages) this gives 64 pages per split, the optimum of a
  // sweep on B200; at 256 x 8 heads it gives one split.
  const int sms = num_sms();
  const long long target = 12ll * sms;
  const long long units = (long long)num_seqs * num_kv_heads;
  const long long splits = units >= target ? 1 : (target + units - 1) / units;
  int pps = (int)((max_blocks_per_seq + splits - 1) / splits);
  pps = (pps + 3) / 4 * 4;
  const int lo = 8 * 16 / block_size > 0 ? 8 * 16 / block_size : 1;  // >= 128 tokens per split
  if (pps < lo) pps = lo;
  if (pps > 128) pps = 128;
  if (pps > max_blocks_per_seq) pps = max_blocks_per_seq;
  *pages_per_split = pps;
  *max_splits = (max_blocks_per_seq + pps - 1) / pps;
  return NB_OK;
}

size_t nb_paged_decode_workspace_size(int num_seqs, int num_q_heads, int head_dim,
                                      int max_splits) {
  if (num_seqs <= 0 || num_q_heads <= 0 || head_dim <= 0 || max_splits <= 1) return 0;
  const size_t n = (size_t)num_seqs * num_q_heads * max_splits;
  return n * head_dim * sizeof(float) + n * sizeof(float2);
}

int nb_paged_decode(const void* q, int64_t q_stride_seq, int64_t q_stride_head,
                    const void* kv_cache, int num_blocks, int num_kv_heads, int block_size,
                    int head_dim, int num_q_heads, const int32_t* block_table,
                    int64_t block_table_stride, int max_blocks_per_seq,
                    const int32_t* context_lens, int num_seqs, float scale, void* out,
                    int64_t out_stride_seq, int64_t out_stride_head, void* workspace,
                    size_t workspace_bytes, int pages_per_split, int dtype, void* stream) {
  using namespace nbh;
  if (!valid_dtype(dtype)) return fail(NB_ERR_INVALID_ARG, "invalid dtype %d", dtype);
  if (!q || !kv_cache || !block_table || !context_lens || !out)
    return fail(NB_ERR_INVALID_ARG, "null pointer argument");
  if (num_blocks <= 0 || num_kv_heads <= 0 || block_size <= 0 || head_dim <= 0 ||
      num_q_heads <= 0 || max_blocks_per_seq <= 0 || num_seqs < 0)
    return fail(NB_ERR_INVALID_ARG, "non-positive shape");
  if (num_q_heads % num_kv_heads)
    return fail(NB_ERR_INVALID_ARG, "num_q_heads %d not a multiple of num_kv_heads %d",
                num_q_heads, num_kv_heads);
  if (block_table_stride < max_blocks_per_seq)
    return fail(NB_ERR_INVALID_ARG, "block_table_stride < max_blocks_per_seq");
  if (pages_per_split <= 0) return fail(NB_ERR_INVALID_ARG, "pages_per_split must be > 0");
  if (head_dim % 32) return fail(NB_ERR_UNSUPPORTED, "head_dim must be a multiple of 32");
  if (q_stride_head < head_dim || out_stride_head < head_dim ||
      q_stride_seq < (int64_t)num_q_heads * q_stride_head - (q_stride_head - head_dim) ||
      out_stride_seq < (int64_t)num_q_heads * out_stride_head - (out_stride_head - head_dim))
    return fail(NB_ERR_INVALID_ARG, "q/out strides overlap");
  if (num_seqs == 0) return NB_OK;
  const int group = num_q_heads / num_kv_heads;
  const int max_splits = (max_blocks_per_seq + pages_per_split - 1) / pages_per_split;
  const size_t need = nb_paged_decode_workspace_size(num_seqs, num_q_heads, head_dim, max_splits);
  if (need > 0 && (!workspace || workspace_bytes < need))
    return fail(NB_ERR_INVALID_ARG, "workspace too small: need %zu bytes, got %zu", need,
                workspace_bytes);
  if ((uintptr_t)workspace % 16) return fail(NB_ERR_INVALID_ARG, "workspace not 16-byte aligned");
  float* po = (float*)workspace;
  float2* pml = need ? (float2*)((char*)workspace +
                                 (size_t)num_seqs * num_q_heads * max_splits * head_dim * 4)
                     : nullptr;
  const float sl2 = scale * nb::kLog2e;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t rows = 2ll * num_blocks * num_kv_heads * block_size;
  const bool tc = dtype != NB_DTYPE_F32 && block_size == 16 &&
                  (head_dim == 64 || head_dim == 128) &&
                  pages_per_split <= max_pages_per_split_tc() && rows < (1ll << 31) &&
                  (uintptr_t)kv_cache % 16 == 0 && (uintptr_t)q % 4 == 0 &&
                  q_stride_seq % 2 == 0 && q_stride_head % 2 == 0;
  int rc;
  if (tc) {
    CUtensorMap map;
    rc = tensor_map_2d(&map, kv_cache, dtype, head_dim, rows, (uint64_t)head_dim * 2, 64, 16);
    if (rc) return rc;
#define NB_ARGS map, q, q_stride_seq, q_stride_head, block_table, block_table_stride,           \
                max_blocks_per_seq, context_lens, num_kv_heads, group, num_blocks, sl2,         \
                pages_per_split, out, out_stride_seq, out_stride_head, po, pml, max_splits,     \
                num_seqs, st
    if (dtype == NB_DTYPE_BF16)
      rc = head_dim == 64 ? dispatch_decode_tc<__nv_bfloat16, 64>(NB_ARGS)
                          : dispatch_decode_tc<__nv_bfloat16, 128>(NB_ARGS);
    else
      rc = head_dim == 64 ? dispatch_decode_tc<__half, 64>(NB_ARGS)
                          : dispatch_decode_tc<__half, 128>(NB_ARGS);
#undef NB_ARGS
  } else {
#define NB_ARGS head_dim, kv_cache, num_blocks, num_kv_heads, block_size, q, q_stride_seq,      \
                q_stride_head, block_table, block_table_stride, max_blocks_per_seq,             \
                context_lens, group, sl2, pages_per_split, out, out_stride_seq,                 \
                out_stride_head, po, pml, max_splits, num_seqs, st
    switch (dtype) {
      case NB_DTYPE_F32: rc = launch_decode_simt_d<float>(NB_ARGS); break;
      case NB_DTYPE_F16: rc = launch_decode_simt_d<__half>(NB_ARGS); break;
      default: rc = launch_decode_simt_d<__nv_bfloat16>(NB_ARGS);
    }
#undef NB_ARGS
  }
  if (rc || max_splits <= 1) return rc;
#define NB_ARGS po, pml, context_lens, max_blocks_per_seq, block_size, pages_per_split, num_seqs, \
                num_q_heads, head_dim, max_splits, out, out_stride_seq, out_stride_head, st
  switch (dtype) {
    case NB_DTYPE_F32: return launch_merge<float>(NB_ARGS);
    case NB_DTYPE_F16: return launch_merge<__half>(NB_ARGS);
    default: return launch_merge<__nv_bfloat16>(NB_ARGS);
  }
#undef NB_ARGS
}

}  // extern "C"
