// Attention backward for sm_100a (B200): dQ, dK, dV of softmax(Q K^T * scale + mask) V.
//
// Replaces the backward nanochat's Blackwell attention op calls,
// _flash_attn_bwd(q, k, v, out, grad_output, lse, causal=True, window_size_left=w)
// (nanochat_autoresearch/solutions/train.py:491,508-519), with the same inputs: the
// forward's output O and its natural-log logsumexp. Math per (batch, head):
//   P = exp(S - lse) with S = Q K^T * scale (masked entries 0)
//   dV = P^T dO      dP = dO V^T      delta = rowsum(dO * O)
//   dS = P * (dP - delta)      dQ = scale dS K      dK = scale dS^T Q
// Grouped-query heads sum into their shared K/V head.
//
// Three launches, no atomics, deterministic:
//   1. attn_bwd_prep_kernel: delta and lse * log2(e) per query row into a workspace,
//      padded to whole 128-row tiles (padding rows: lse2 = +inf, delta = 0, so they
//      contribute exactly 0 everywhere).
//   2. attn_bwd_sm100_kernel<KV = true>: one work item per (batch, K/V head, 128-key
//      block); K and V stay in shared memory while the item streams (Q, dO) tiles of every
//      query head of the group:
//        T1 = S^T = K Q^T,  T2 = dP^T = V dO^T           (tcgen05.mma, both K-major)
//        P^T, dS^T from T1, T2 (softmax warps, thread = key row)
//        dV += P^T dO,  dK += dS^T Q                      (A operand read from TMEM)
//   3. attn_bwd_sm100_kernel<KV = false>: one item per (batch, query head, 128-row block);
//      Q and dO stay resident while K, V tiles stream:
//        T1 = S = Q K^T,  T2 = dP = dO V^T,  dS,  dQ += dS K.
// The dQ pass recomputes S and dP (3 GEMMs per tile) instead of accumulating dQ with
// atomics from the dK/dV pass, trading 40% more tensor work for deterministic results and
// no fp32 dQ scratch.
//
// In both passes P and dS are written back into the TMEM columns of the scores they came
// from, packed as 16-bit pairs, and read from there as the A operand of the accumulating
// MMAs, so the only shared-memory traffic is the TMA tiles.
//
// Warp roles (320 threads): warps 0-7 elementwise (warpgroup h handles columns
// [64h, 64h + 64) of the 128 x 128 tile, a half with its own barriers, so the two halves
// pipeline against each other's MMAs; thread = TMEM lane = row) and the per-item epilogue;
// warp 8 issues every MMA (and owns TMEM); warp 9 schedules items and issues TMA.
#pragma once

#include "attn_fwd_kernel.cuh"

namespace apex {

struct BwdParams {
  void* out1;            // dK (KV pass) or dQ (Q pass)
  void* out2;            // dV (KV pass)
  long long o1_sb, o1_sh, o1_sn;
  long long o2_sb, o2_sh, o2_sn;
  const float* lse2;     // workspace [B * H][Npad]: lse * log2(e), +inf on padding rows
  const float* delta;    // workspace [B * H][Npad]: rowsum(dO * O), 0 on padding rows
  int* status;
  int* work_counter;
  int B, H, Hkv, N, Npad;
  int nblk;              // ceil(N / 128)
  int num_items;
  int group_q, group_big;  // L2 scheduling groups over the item heads (as in the forward)
  int kv_group;          // H / Hkv
  float scale_log2;      // sm_scale * log2(e)
  float out1_scale;      // sm_scale (dK = scale dS^T Q, dQ = scale dS K)
  int causal;
  int window;            // -1: none
  unsigned long long timeout_ns;
};

template <int D>
struct BwdCfg {
  static_assert(D == 64 || D == 128, "backward head dims 64, 128");
  static constexpr int kNS = D == 64 ? 8 : 4;  // streaming ring stages (one 128-row tile each)
  static constexpr int kThreads = 320;
  static constexpr int kWarpMma = 8;
  static constexpr int kWarpProd = 9;
  // TMEM columns: T1 scores, T2 dP, Acc1 dK | dQ, Acc2 dV.
  static constexpr int kT1 = 0;
  static constexpr int kT2 = 128;
  static constexpr int kAcc1 = 256;
  static constexpr int kAcc2 = 256 + D;
  static_assert(kAcc2 + D <= 512, "TMEM plan overflows 512 columns");
};

template <int D>
struct BwdSmem {
  using C = BwdCfg<D>;
  static constexpr int NS = C::kNS;
  static constexpr int kChunkBytes = kBlockM * 128;
  static constexpr int kTileBytes = kBlockM * D * 2;
  static constexpr int kX1 = 0;
  static constexpr int kX2 = kX1 + kTileBytes;
  static constexpr int kRing = kX2 + kTileBytes;
  static constexpr int kStats = kRing + NS * kTileBytes;  // float [NS][256]: lse2[128], delta[128]
  static constexpr int kStatsBytes = 1024;
  static constexpr int kBars = kStats + NS * kStatsBytes;
  static constexpr int kRingFull = 0;
  static constexpr int kRingEmpty = NS;
  static constexpr int kXFull = 2 * NS;
  static constexpr int kXEmpty = kXFull + 1;
  // Per column half h of the 128 x 128 tile (two slots each):
  static constexpr int kT1Full = kXEmpty + 1;  // [2] scores of half h in TMEM
  static constexpr int kT2Full = kT1Full + 2;  // [2] dP of half h in TMEM
  static constexpr int kPFull = kT2Full + 2;   // [2] P of half h packed in TMEM (KV pass)
  static constexpr int kDSFull = kPFull + 2;   // [2] dS of half h packed in TMEM
  static constexpr int kTFree = kDSFull + 2;   // [2] accumulating MMAs of half h done
  static constexpr int kAccFull = kTFree + 2;
  static constexpr int kAccEmpty = kAccFull + 1;
  static constexpr int kDrain = kAccEmpty + 1;
  static constexpr int kItemFull = kDrain + 1;
  static constexpr int kItemEmpty = kItemFull + kItemRing;
  static constexpr int kNumBars = kItemEmpty + kItemRing;
  static constexpr int kItems = kBars + kNumBars * 8;
  static constexpr int kMisc = kItems + kItemRing * 4;  // tmem base, abort flag
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kDynamicBytes = kBytes + 1024;
  static_assert(kDynamicBytes <= 232448, "shared-memory plan exceeds 227 KB");
};

// One work item: the stationary 128-row block `blk` of head `hx` (K/V head in the KV pass,
// query head in the Q pass) and the range [lo, hi) of streaming tiles it meets (query tiles
// in the KV pass, repeated for each of the kv_group query heads; key blocks in the Q pass).
struct BwdItem {
  int b, hx, blk, lo, hi, nsteps;
};

// Item t -> work, longest first inside equal-size L2 groups of heads (see decode_item).
template <bool KV, bool WIN>
__device__ __forceinline__ BwdItem decode_bwd(int t, const BwdParams& p) {
  const int MB = p.nblk;
  const int q = p.group_q;
  const int big_items = p.group_big * (q + 1) * MB;
  int size, base, r;
  if (t < big_items) {
    size = q + 1;
    const int g = t / (size * MB);
    r = t - g * size * MB;
    base = g * size;
  } else {
    size = q;
    const int t2 = t - big_items;
    const int g = t2 / (size * MB);
    r = t2 - g * size * MB;
    base = p.group_big * (q + 1) + g * size;
  }
  const int rb = r / size;
  const int bh = base + r % size;
  const int HX = KV ? p.Hkv : p.H;
  BwdItem it;
  it.b = bh / HX;
  it.hx = bh - it.b * HX;
  if (KV) {
    // Causal: key block blk is seen by query tiles >= blk, so low blocks are the long ones.
    it.blk = rb;
    it.lo = p.causal ? it.blk : 0;
    it.hi = p.nblk;
    if (WIN) it.hi = min(p.nblk, (it.blk * kBlockN + kBlockN - 1 + p.window) / kBlockM + 1);
    it.nsteps = p.kv_group * (it.hi - it.lo);
  } else {
    it.blk = MB - 1 - rb;
    it.lo = WIN ? max(0, it.blk * kBlockM - p.window) / kBlockN : 0;
    it.hi = p.causal ? it.blk + 1 : p.nblk;
    it.nsteps = it.hi - it.lo;
  }
  return it;
}

// delta[bh][i] = sum_d dO[b,h,i,d] O[b,h,i,d] (fp32) and lse2[bh][i] = lse[bh][i] log2(e),
// for i < Npad (padding rows: delta 0, lse2 +inf). kTpr = D / 8 threads per row, each
// reading one 16-byte vector of O and of dO.
template <typename T, int D>
__global__ void __launch_bounds__(256) attn_bwd_prep_kernel(const T* __restrict__ o,
                                                            const T* __restrict__ dout,
                                                            const float* __restrict__ lse,
                                                            float* __restrict__ lse2,
                                                            float* __restrict__ delta, long long o_sb,
                                                            long long o_sh, long long o_sn,
                                                            long long d_sb, long long d_sh,
                                                            long long d_sn, int H, int N, int Npad,
                                                            long long rows) {
  constexpr int kTpr = D / 8;
  const long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) / kTpr;
  const int sub = (int)(threadIdx.x % kTpr);
  const bool in_range = row < rows;  // no early exit: every lane takes part in the shuffles
  const int i = in_range ? (int)(row % Npad) : 0;
  const long long bh = in_range ? row / Npad : 0;
  const int b = (int)(bh / H);
  const int h = (int)(bh - (long long)b * H);
  float acc = 0.f;
  if (in_range && i < N) {
    const uint4 a = *reinterpret_cast<const uint4*>(o + b * o_sb + h * o_sh + i * o_sn + sub * 8);
    const uint4 g = *reinterpret_cast<const uint4*>(dout + b * d_sb + h * d_sh + i * d_sn + sub * 8);
    const T* av = reinterpret_cast<const T*>(&a);
    const T* gv = reinterpret_cast<const T*>(&g);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc = fmaf((float)av[e], (float)gv[e], acc);
  }
#pragma unroll
  for (int w = kTpr / 2; w > 0; w >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, w);
  if (in_range && sub == 0) {
    delta[row] = acc;
    lse2[row] = i < N ? lse[bh * N + i] * 1.4426950408889634f : INFINITY;
  }
}

// KV = true: dK, dV pass; KV = false: dQ pass. WIN: causal sliding window in use.
template <int D, typename T, bool KV, bool WIN>
__global__ void __launch_bounds__(BwdCfg<D>::kThreads, 1)
    attn_bwd_sm100_kernel(const __grid_constant__ CUtensorMap tmX1,
                          const __grid_constant__ CUtensorMap tmX2,
                          const __grid_constant__ CUtensorMap tmY1,
                          const __grid_constant__ CUtensorMap tmY2, const BwdParams p) {
  using C = BwdCfg<D>;
  using Plan = BwdSmem<D>;
  constexpr int NS = C::kNS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  const uint32_t sbase = raw_addr + pad;
  uint8_t* smem = smem_raw + pad;

  const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0);
  const int lane = (int)(threadIdx.x & 31);
  auto bar = [&](int slot) -> uint32_t { return sbase + Plan::kBars + slot * 8; };
  int* items = reinterpret_cast<int*>(smem + Plan::kItems);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Plan::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Plan::kMisc + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      ptx::mbar_init(bar(Plan::kRingFull + s), 1);
      ptx::mbar_init(bar(Plan::kRingEmpty + s), 1);
    }
    ptx::mbar_init(bar(Plan::kXFull), 1);
    ptx::mbar_init(bar(Plan::kXEmpty), 1);
    for (int h = 0; h < 2; ++h) {
      ptx::mbar_init(bar(Plan::kT1Full + h), 1);
      ptx::mbar_init(bar(Plan::kT2Full + h), 1);
      ptx::mbar_init(bar(Plan::kPFull + h), 128);
      ptx::mbar_init(bar(Plan::kDSFull + h), 128);
      ptx::mbar_init(bar(Plan::kTFree + h), 1);
    }
    ptx::mbar_init(bar(Plan::kAccFull), 1);
    ptx::mbar_init(bar(Plan::kAccEmpty), 256);
    ptx::mbar_init(bar(Plan::kDrain), 1);
    // Item-ring readers: the 8 elementwise warps and the MMA warp.
    for (int k = 0; k < kItemRing; ++k) {
      ptx::mbar_init(bar(Plan::kItemFull + k), 1);
      ptx::mbar_init(bar(Plan::kItemEmpty + k), 9);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == C::kWarpMma) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), 512);
    ptx::tmem_relinquish();
  }
  if (warp == C::kWarpProd && lane == 0) {
    ptx::prefetch_tmap(&tmX1);
    ptx::prefetch_tmap(&tmX2);
    ptx::prefetch_tmap(&tmY1);
    ptx::prefetch_tmap(&tmY2);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const Waiter W{abort_flag, p.status, p.timeout_ns};

  if (warp < C::kWarpMma) {
    // ======================================================== elementwise ===
    const int quarter = warp & 3;
    const int half = warp >> 2;          // column half of the 128 x 128 tile
    const int r = quarter * 32 + lane;   // row (TMEM lane)
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tT1 = tmem + lane_off + (uint32_t)(C::kT1 + 64 * half);
    const uint32_t tT2 = tmem + lane_off + (uint32_t)(C::kT2 + 64 * half);
    const float* stats = reinterpret_cast<const float*>(smem + Plan::kStats);
    const float c = p.scale_log2;
    Ring<NS> ring;
    uint32_t t1_par = 0, t2_par = 0, af_par = 0;
    bool ok = true;
    ItemReader reader;
    while (ok) {
      int t;
      if (!(ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, true, t)) || t < 0) break;
      const BwdItem it = decode_bwd<KV, WIN>(t, p);
      const int nq = it.hi - it.lo;
      // Q pass: this thread's query row statistics, fixed for the item.
      float row_lse2 = 0.f, row_delta = 0.f;
      if (!KV) {
        const long long idx = ((long long)it.b * p.H + it.hx) * p.Npad + it.blk * kBlockM + r;
        row_lse2 = p.lse2[idx];
        row_delta = p.delta[idx];
      }
      for (int s = 0; s < it.nsteps && ok; ++s) {
        const int ytile = it.lo + (KV ? s % nq : s);
        // KV pass: the stage holding this step's Q tile also holds its lse2/delta.
        const int st1 = ring.stage;
        const uint32_t ph1 = ring.phase;
        ring.next();
        ring.next();
        const float* st_lse = stats + st1 * 256 + 64 * half;
        const float* st_delta = st_lse + 128;
        if (KV && !(ok = W.wait_warp(bar(Plan::kRingFull + st1), ph1))) break;
        // Mask geometry: qi - kj = dq0 + (KV ? col - row : row - col).
        const int it_q = KV ? ytile : it.blk;
        const int jb_k = KV ? it.blk : ytile;
        const int dq0 = (it_q - jb_k) * kBlockM;
        const bool masked = (p.causal && it_q == jb_k) || (WIN && dq0 + kBlockM - 1 > p.window);
        const int colbase = 64 * half;
        if (!(ok = W.wait_warp(bar(Plan::kT1Full + half), t1_par))) break;
        t1_par ^= 1;
        ptx::tc_fence_after();
        float pv[64];
        {
          uint32_t v[2][32];
          ptx::tmem_ld32(tT1, v[0]);
          ptx::tmem_ld32(tT1 + 32, v[1]);
          ptx::tmem_wait_ld();
          ptx::reg_fence32(v[0]);
          ptx::reg_fence32(v[1]);
          if (KV) {
#pragma unroll
            for (int e = 0; e < 64; e += 4) {
              const float4 l4 = *reinterpret_cast<const float4*>(st_lse + e);
              const float2 x0 = __ffma2_rn(make_float2(__uint_as_float(v[e >> 5][e & 31]), __uint_as_float(v[e >> 5][(e & 31) + 1])),
                                           make_float2(c, c), make_float2(-l4.x, -l4.y));
              const float2 x1 = __ffma2_rn(make_float2(__uint_as_float(v[e >> 5][(e & 31) + 2]), __uint_as_float(v[e >> 5][(e & 31) + 3])),
                                           make_float2(c, c), make_float2(-l4.z, -l4.w));
              pv[e] = x0.x;
              pv[e + 1] = x0.y;
              pv[e + 2] = x1.x;
              pv[e + 3] = x1.y;
            }
          } else {
            const float2 nl = make_float2(-row_lse2, -row_lse2);
#pragma unroll
            for (int e = 0; e < 64; e += 2) {
              const float2 x = __ffma2_rn(make_float2(__uint_as_float(v[e >> 5][e & 31]), __uint_as_float(v[e >> 5][(e & 31) + 1])),
                                          make_float2(c, c), nl);
              pv[e] = x.x;
              pv[e + 1] = x.y;
            }
          }
        }
        if (masked) {
#pragma unroll
          for (int e = 0; e < 64; ++e) {
            const int dqk = dq0 + (KV ? colbase + e - r : r - colbase - e);
            if ((p.causal && dqk < 0) || (WIN && dqk > p.window)) pv[e] = -INFINITY;
          }
        }
#pragma unroll
        for (int e = 0; e < 64; ++e) pv[e] = ptx::ex2(pv[e]);  // masked: exactly 0
        if (KV) {
          // P^T packed into this warpgroup's first 32 T1 columns: the A operand of dV.
          uint32_t pk[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) pk[e] = DType<T>::pack(pv[2 * e], pv[2 * e + 1]);
          ptx::tmem_st32(tT1, pk);
          ptx::tmem_wait_st();
          ptx::tc_fence_before();
          ptx::mbar_arrive(bar(Plan::kPFull + half));
        }
        if (!(ok = W.wait_warp(bar(Plan::kT2Full + half), t2_par))) break;
        t2_par ^= 1;
        ptx::tc_fence_after();
        {
          uint32_t v[2][32];
          ptx::tmem_ld32(tT2, v[0]);
          ptx::tmem_ld32(tT2 + 32, v[1]);
          ptx::tmem_wait_ld();
          ptx::reg_fence32(v[0]);
          ptx::reg_fence32(v[1]);
          uint32_t pk[32];
          if (KV) {
#pragma unroll
            for (int e = 0; e < 64; e += 4) {
              const float4 d4 = *reinterpret_cast<const float4*>(st_delta + e);
              const float a0 = pv[e] * (__uint_as_float(v[e >> 5][e & 31]) - d4.x);
              const float a1 = pv[e + 1] * (__uint_as_float(v[e >> 5][(e & 31) + 1]) - d4.y);
              const float a2 = pv[e + 2] * (__uint_as_float(v[e >> 5][(e & 31) + 2]) - d4.z);
              const float a3 = pv[e + 3] * (__uint_as_float(v[e >> 5][(e & 31) + 3]) - d4.w);
              pk[e >> 1] = DType<T>::pack(a0, a1);
              pk[(e >> 1) + 1] = DType<T>::pack(a2, a3);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 64; e += 2) {
              const float a0 = pv[e] * (__uint_as_float(v[e >> 5][e & 31]) - row_delta);
              const float a1 = pv[e + 1] * (__uint_as_float(v[e >> 5][(e & 31) + 1]) - row_delta);
              pk[e >> 1] = DType<T>::pack(a0, a1);
            }
          }
          // dS packed into this warpgroup's first 32 T2 columns: the A operand of dK / dQ.
          ptx::tmem_st32(tT2, pk);
          ptx::tmem_wait_st();
        }
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(Plan::kDSFull + half));
      }
      if (!ok) break;
      // ---- epilogue: Acc1 * scale -> out1 (dK | dQ), Acc2 -> out2 (dV) ----
      if (!(ok = W.wait_warp(bar(Plan::kAccFull), af_par))) break;
      af_par ^= 1;
      ptx::tc_fence_after();
      const int row = it.blk * kBlockM + r;
      const bool valid = row < p.N;
      constexpr int kHalfCols = D / 2;
      auto store = [&](void* base, long long sb, long long sh, long long sn, int acc_col, float scale) {
        T* dst = reinterpret_cast<T*>(base) + (long long)it.b * sb + (long long)it.hx * sh +
                 (long long)row * sn + half * kHalfCols;
#pragma unroll 1
        for (int ch = 0; ch < kHalfCols / 32; ++ch) {
          uint32_t v[32];
          ptx::tmem_ld32(tmem + lane_off + (uint32_t)(acc_col + half * kHalfCols + ch * 32), v);
          ptx::tmem_wait_ld();
          ptx::reg_fence32(v);
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            pk[e] = DType<T>::pack(__uint_as_float(v[2 * e]) * scale, __uint_as_float(v[2 * e + 1]) * scale);
          if (valid) {
            uint4* d4 = reinterpret_cast<uint4*>(dst + ch * 32);
#pragma unroll
            for (int w = 0; w < 4; ++w) d4[w] = make_uint4(pk[4 * w], pk[4 * w + 1], pk[4 * w + 2], pk[4 * w + 3]);
          }
        }
      };
      store(p.out1, p.o1_sb, p.o1_sh, p.o1_sn, C::kAcc1, p.out1_scale);
      if (KV) store(p.out2, p.o2_sb, p.o2_sh, p.o2_sn, C::kAcc2, 1.f);
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar(Plan::kAccEmpty));
    }
  } else if (warp == C::kWarpMma) {
    // ================================================================ MMA ===
    // Each 128 x 128 step is issued as two column halves h (64 streaming rows each), so
    // the tensor pipe works on one half while the elementwise warpgroup of the other
    // half runs. Issue order per step s:
    //   G1_0 G2_0 G1_1 G2_1 | G3_0 G4_0 G3_1 G4_1
    // with G1_h: T1_h = X1 Y1_h^T, G2_h: T2_h = X2 Y2_h^T (128 x 64 x D each), G3_h: Acc2 +=
    // P_h Y2_h (KV pass), G4_h: Acc1 += dS_h Y1_h (128 x D x 64 each). G1_h/G2_h of step s+1
    // wait only for G3_h/G4_h of step s (TFree_h), which were issued before G3/G4 of the
    // other half, so the pipe never drains between steps.
    constexpr uint32_t idNT = make_idesc<T>(kBlockM, 64, false);  // T_h = X Y_h^T
    constexpr uint32_t idAcc = make_idesc<T>(kBlockM, D, true);   // Acc += A_h(TMEM) Y_h
    constexpr uint32_t kHalfRows = 64 * 128;  // byte offset of row 64 inside a 128-row chunk
    const uint32_t sX1 = sbase + Plan::kX1;
    const uint32_t sX2 = sbase + Plan::kX2;
    const uint32_t sRing = sbase + Plan::kRing;
    auto gemm_nt = [&](uint32_t d_tmem, uint32_t sA, uint32_t sB) {
      const uint64_t a0 = make_sdesc_sw128(sA, 16, 1024);
      const uint64_t b0 = make_sdesc_sw128(sB, 16, 1024);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (uint32_t)((kk >> 2) * Plan::kChunkBytes + (kk & 3) * 32) >> 4;
        ptx::umma_ss_warp(d_tmem, a0 + off, b0 + off, idNT, kk > 0 ? 1u : 0u);
      }
    };
    // A: 128 x 64 16-bit operand packed in 32 TMEM columns at a_tmem; B: 64 rows x D.
    auto gemm_acc = [&](uint32_t d_tmem, uint32_t a_tmem, uint32_t sB, bool accumulate) {
      const uint64_t b0 = make_sdesc_sw128(sB, Plan::kChunkBytes, 1024);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t boff = (uint32_t)(kk * 16 * 128) >> 4;
        ptx::umma_ts_warp(d_tmem, a_tmem + (uint32_t)(8 * kk), b0 + boff, idAcc,
                          (accumulate || kk > 0) ? 1u : 0u);
      }
    };
    const uint32_t tAcc1 = tmem + C::kAcc1, tAcc2 = tmem + C::kAcc2;
    Ring<NS> ring;
    uint32_t x_par = 0, tf_par = 0, pf_par = 0, df_par = 0, ae_par = 0;  // bit h: half h
    int steps_done = 0, items_done = 0;
    bool ok = true;
    auto acquire = [&]() -> int {
      const int st = ring.stage;
      const uint32_t ph = ring.phase;
      ring.next();
      if (!W.wait_warp(bar(Plan::kRingFull + st), ph)) return -1;
      ptx::tc_fence_after();
      return st;
    };
    auto wait_bit = [&](int slot, uint32_t& par, int h) -> bool {
      if (!W.wait_warp(bar(slot + h), (par >> h) & 1u)) return false;
      par ^= 1u << h;
      ptx::tc_fence_after();
      return true;
    };
    ItemReader reader;
    while (ok) {
      int t;
      if (!(ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, true, t)) || t < 0) break;
      const BwdItem it = decode_bwd<KV, WIN>(t, p);
      if (!(ok = W.wait_warp(bar(Plan::kXFull), x_par))) break;
      x_par ^= 1;
      ptx::tc_fence_after();
      for (int s = 0; s < it.nsteps && ok; ++s) {
        const int st1 = acquire();
        ok = st1 >= 0;
        if (!ok) break;
        const int st2 = acquire();
        ok = st2 >= 0;
        if (!ok) break;
        const uint32_t sY1 = sRing + st1 * Plan::kTileBytes;
        const uint32_t sY2 = sRing + st2 * Plan::kTileBytes;
#pragma unroll 1
        for (int h = 0; h < 2 && ok; ++h) {
          // T1_h, T2_h still hold P_h / dS_h of the previous step until its G3_h/G4_h finish.
          if (steps_done > 0 && !(ok = wait_bit(Plan::kTFree, tf_par, h))) break;
          gemm_nt(tmem + (uint32_t)(C::kT1 + 64 * h), sX1, sY1 + h * kHalfRows);
          ptx::tc_commit_warp(bar(Plan::kT1Full + h));
          gemm_nt(tmem + (uint32_t)(C::kT2 + 64 * h), sX2, sY2 + h * kHalfRows);
          ptx::tc_commit_warp(bar(Plan::kT2Full + h));
        }
        if (!ok) break;
        if (s == it.nsteps - 1) ptx::tc_commit_warp(bar(Plan::kXEmpty));  // last reads of X1, X2
        if (!KV) ptx::tc_commit_warp(bar(Plan::kRingEmpty + st2));        // V: only dP reads it
        if (s == 0 && items_done > 0) {  // the epilogue must have drained the accumulators
          if (!(ok = W.wait_warp(bar(Plan::kAccEmpty), ae_par))) break;
          ae_par ^= 1;
          ptx::tc_fence_after();
        }
#pragma unroll 1
        for (int h = 0; h < 2 && ok; ++h) {
          const bool acc = s > 0 || h > 0;
          if (KV) {
            if (!(ok = wait_bit(Plan::kPFull, pf_par, h))) break;
            gemm_acc(tAcc2, tmem + (uint32_t)(C::kT1 + 64 * h), sY2 + h * kHalfRows, acc);  // dV += P^T dO
          }
          if (!(ok = wait_bit(Plan::kDSFull, df_par, h))) break;
          gemm_acc(tAcc1, tmem + (uint32_t)(C::kT2 + 64 * h), sY1 + h * kHalfRows, acc);  // dK | dQ
          ptx::tc_commit_warp(bar(Plan::kTFree + h));
        }
        if (!ok) break;
        if (KV) ptx::tc_commit_warp(bar(Plan::kRingEmpty + st2));
        ptx::tc_commit_warp(bar(Plan::kRingEmpty + st1));
        ++steps_done;
      }
      if (!ok) break;
      ptx::tc_commit_warp(bar(Plan::kAccFull));
      ++items_done;
    }
    ptx::tc_commit_warp(bar(Plan::kDrain));
    if (lane == 0) drain_wait(bar(Plan::kDrain), 0, p.timeout_ns, p.status);
    __syncwarp();
  } else {
    // ============================================== scheduler + producer ===
    if (lane == 0) {
      const uint64_t pol_x = ptx::policy_evict_first();  // read by this item only
      const uint64_t pol_y = ptx::policy_evict_last();   // re-read by every block of the head
      const uint32_t sX1 = sbase + Plan::kX1;
      const uint32_t sX2 = sbase + Plan::kX2;
      const uint32_t sRing = sbase + Plan::kRing;
      const uint32_t sStats = sbase + Plan::kStats;
      Ring<NS> ring;
      uint32_t xe_par = 1;
      int fills = 0, x_fills = 0;
      bool ok = true;
      auto load_tile = [&](uint32_t dst, const CUtensorMap* map, uint32_t b, int row0, int h, int bi,
                           uint64_t pol) {
#pragma unroll
        for (int cc = 0; cc < D / 64; ++cc)
          ptx::tma_load_4d(dst + cc * Plan::kChunkBytes, map, b, cc * 64, row0, h, bi, pol);
      };
      int fetched = atomicAdd(p.work_counter, 1);
      int published = 0;
      while (ok) {
        const int slot = published % kItemRing;
        const uint32_t parity = ((uint32_t)(published / kItemRing) & 1u) ^ 1u;
        if (!(ok = W.wait(bar(Plan::kItemEmpty + slot), parity))) break;
        const int t = fetched < p.num_items ? fetched : -1;
        if (t >= 0) fetched = atomicAdd(p.work_counter, 1);
        items[slot] = t;
        ptx::mbar_arrive(bar(Plan::kItemFull + slot));
        ++published;
        if (t < 0) break;
        const BwdItem it = decode_bwd<KV, WIN>(t, p);
        if (!(ok = W.wait(bar(Plan::kXEmpty), xe_par))) break;
        xe_par ^= 1;
        ptx::mbar_arrive_expect_tx(bar(Plan::kXFull), 2u * Plan::kTileBytes);
        load_tile(sX1, &tmX1, bar(Plan::kXFull), it.blk * kBlockM, it.hx, it.b, pol_x);
        load_tile(sX2, &tmX2, bar(Plan::kXFull), it.blk * kBlockM, it.hx, it.b, pol_x);
        ++x_fills;
        const int nq = it.hi - it.lo;
        for (int s = 0; s < it.nsteps && ok; ++s) {
          const int ytile = it.lo + (KV ? s % nq : s);
          const int hy = KV ? it.hx * p.kv_group + s / nq : it.hx / p.kv_group;
          for (int k = 0; k < 2; ++k) {
            const int st = ring.stage;
            const uint32_t ph = ring.phase;
            ring.next();
            if (!(ok = W.wait(bar(Plan::kRingEmpty + st), ph ^ 1))) break;
            const bool with_stats = KV && k == 0;
            ptx::mbar_arrive_expect_tx(bar(Plan::kRingFull + st),
                                       (uint32_t)Plan::kTileBytes + (with_stats ? 1024u : 0u));
            load_tile(sRing + st * Plan::kTileBytes, k == 0 ? &tmY1 : &tmY2, bar(Plan::kRingFull + st),
                      ytile * kBlockN, hy, it.b, pol_y);
            if (with_stats) {
              const long long idx = ((long long)it.b * p.H + hy) * p.Npad + (long long)ytile * kBlockM;
              ptx::bulk_load(sStats + st * Plan::kStatsBytes, p.lse2 + idx, 512u, bar(Plan::kRingFull + st), pol_y);
              ptx::bulk_load(sStats + st * Plan::kStatsBytes + 512, p.delta + idx, 512u, bar(Plan::kRingFull + st), pol_y);
            }
            ++fills;
          }
        }
      }
      // Let every load this thread issued land before the CTA exits.
      const int last = fills < NS ? fills : NS;
      for (int k = 0; k < last; ++k) {
        const int f = fills - 1 - k;
        drain_wait(bar(Plan::kRingFull + (f % NS)), (uint32_t)((f / NS) & 1), p.timeout_ns, p.status);
      }
      if (x_fills > 0) drain_wait(bar(Plan::kXFull), (uint32_t)((x_fills - 1) & 1), p.timeout_ns, p.status);
    }
    __syncwarp();
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == C::kWarpMma) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

}  // namespace apex
