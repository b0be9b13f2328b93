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
// TMEM and scheduling (both passes, 128 x 128 tiles, one CTA per SM):
//   T1 [0, 128)     scores S^T | S (fp32). The elementwise warps read them into registers
//                   and release T1 at once, so the next step's score GEMM overlaps the
//                   exponentials of this one.
//   T2 [128, 256)   dP^T | dP (fp32); after the elementwise pass it holds the 16-bit
//                   operands of the accumulating GEMMs, packed two per column: warpgroup h
//                   writes P_h (KV pass) and dS_h into its own 64 columns.
//   Acc1, Acc2      dK and dV (KV pass) or dQ (Q pass), fp32, for the whole item.
//   X (Q pass)      Q and dO of the item, copied from shared memory into the 128 free
//                   columns, so the score GEMMs read A from TMEM and only B (K, V tiles)
//                   from shared memory.
// The MMA warp runs a software pipeline: G1(s+1) (scores) is issued once the elementwise
// warps hold S(s), then the accumulating GEMMs of step s, then G2(s+1) (dP), whose
// target T2 becomes free when those complete. A 128 x 128 x 16 MMA whose A and B both come
// from shared memory reads 8 KB, the shared-memory bandwidth of its 64 tensor cycles, so
// every GEMM here is at least 128 wide in N.
//
// Warp roles (384 threads): warps 0-7 elementwise (warpgroup h handles columns
// [64h, 64h + 64) of the 128 x 128 tile; thread = TMEM lane = row) and the per-item
// epilogue; warp 8 issues every MMA (and owns TMEM); warp 9 schedules items and issues TMA;
// warps 10-11 only give their registers to the elementwise warpgroups.
#pragma once

#include "attn_fwd_kernel.cuh"

#ifndef APEX_BWD_SPLIT_DP_KV
#define APEX_BWD_SPLIT_DP_KV 1
#endif
// Of every 8 pairs of exponentials in an unmasked tile, how many the elementwise warps take
// from the FMA-pipe polynomial (exp2_poly_pair) instead of MUFU ex2, per head dim. Both
// warpgroups run their exponentials at the same time, which is MUFU-bound (16 per clock per
// SM) while the FMA pipe idles. Measured with both builds alternating call by call in one
// process: at d = 64 two pairs in eight take the C2 backward from 0.627 to 0.603 ms (one
// pair: 0.621); at d = 128 one or two pairs are within run-to-run noise (6.74-6.82 ms).
#ifndef APEX_BWD_EMU64
#define APEX_BWD_EMU64 2
#endif
#ifndef APEX_BWD_EMU128
#define APEX_BWD_EMU128 0
#endif

namespace apex {

struct BwdParams {
  void* out1;            // dK (KV pass) or dQ (Q pass)
  void* out2;            // dV (KV pass)
  long long o1_sb, o1_sh, o1_sn;
  long long o2_sb, o2_sh, o2_sn;
  const float* nlse2;    // workspace [B * H][Npad]: -lse * log2(e), -inf on padding rows
  const float* ndelta;   // workspace [B * H][Npad]: -rowsum(dO * O), 0 on padding rows
  int* status;
  int* host_flag;  // nullable: mapped pinned host word set to 1 with any status bit
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
  // Packed variable-length batch (VAR kernels): sequence b is rows
  // [cu_seqlens[b], cu_seqlens[b + 1]) of tensors with `total` rows, N is the longest
  // sequence; the statistics stay [B][H][Npad] (per sequence, padded). Offsets are
  // clamped to [0, total] and lengths to N on the device.
  const int* cu_seqlens;
  int total;
  unsigned long long timeout_ns;
};

template <int D>
struct BwdCfg {
  static_assert(D == 64 || D == 128, "backward head dims 64, 128");
  // Streaming ring stages (one 128-row tile each). A stage frees when the accumulating GEMMs
  // of its step finish and takes ~1300 cycles to refill from L2, so the ring holds about
  // two and a half steps (two tiles per step).
  static constexpr int kNS = D == 64 ? 10 : 5;
  // 12 warps: 8 elementwise, MMA, producer, 2 idle. Registers are granted per warpgroup,
  // so the launch budget is 384 x 168; setmaxnreg moves it to the elementwise warpgroups
  // (the split must not exceed the launch allocation, or setmaxnreg.inc would never return).
  static constexpr int kThreads = 384;
  static constexpr int kWarpMma = 8;
  static constexpr int kWarpProd = 9;
  static constexpr int kRegsElementwise = 224;
  static constexpr int kRegsOther = 56;
  static constexpr int kLaunchRegs = (65536 / kThreads) / 8 * 8;
  static_assert(128 * (2 * kRegsElementwise + kRegsOther) <= kThreads * kLaunchRegs,
                "setmaxnreg split exceeds the launch register allocation");
  // TMEM columns: T1 scores, T2 dP (then packed P / dS), Acc1 dK | dQ, Acc2 dV (KV pass),
  // XQ / XdO the item's Q and dO as 16-bit pairs (Q pass).
  static constexpr int kT1 = 0;
  static constexpr int kT2 = 128;
  static constexpr int kAcc1 = 256;
  static constexpr int kAcc2 = 256 + D;
  static constexpr int kXQ = 256 + D;
  static constexpr int kXdO = kXQ + D / 2;
  static_assert(kAcc2 + D <= 512 && kXdO + D / 2 <= 512, "TMEM plan overflows 512 columns");
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
  // KV pass: per-column statistics of the step's query tile, double-buffered:
  // float [2][256] = -lse2[128], -delta[128].
  static constexpr int kStats = kRing + NS * kTileBytes;
  static constexpr int kStatsBytes = 1024;
  static constexpr int kBars = kStats + 2 * kStatsBytes;
  static constexpr int kRingFull = 0;
  static constexpr int kRingEmpty = NS;
  static constexpr int kXFull = 2 * NS;         // X tiles of the item landed in shared memory
  static constexpr int kXEmpty = kXFull + 1;    // shared-memory X may be refilled
  static constexpr int kXTFull = kXEmpty + 1;   // Q pass: X copied into TMEM
  static constexpr int kXTFree = kXTFull + 1;   // Q pass: last MMA reading TMEM X done
  static constexpr int kT1Full = kXTFree + 1;
  static constexpr int kT1Free = kT1Full + 1;   // elementwise warps hold S in registers
  static constexpr int kT2Full = kT1Free + 1;   // [2] dP of column half h
  static constexpr int kT2Free = kT2Full + 2;   // [2] accumulating GEMMs of half h done
  static constexpr int kPdSFull = kT2Free + 2;  // [2] P_h / dS_h packed in T2
  static constexpr int kStatsFull = kPdSFull + 2;    // [2]
  static constexpr int kStatsEmpty = kStatsFull + 2;  // [2]
  static constexpr int kAccFull = kStatsEmpty + 2;
  static constexpr int kAccEmpty = kAccFull + 1;
  static constexpr int kDrain = kAccEmpty + 1;
  static constexpr int kItemFull = kDrain + 1;
  static constexpr int kItemEmpty = kItemFull + kItemRing;
  static constexpr int kNumBars = kItemEmpty + kItemRing;
  static constexpr int kItems = kBars + kNumBars * 8;
  static constexpr int kMisc = kItems + kItemRing * 4;  // tmem base, abort flag
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kMaxDynamic = 232448;  // 227 KB per CTA on sm_100
  // 1 KB of alignment slack when it fits; otherwise the kernel relies on the dynamic shared
  // memory base being 1 KB aligned and checks it (as the forward does).
  static constexpr int kDynamicBytes = kBytes + 1024 <= kMaxDynamic ? kBytes + 1024 : kBytes;
  static_assert(kBytes <= kMaxDynamic, "shared-memory plan exceeds 227 KB");
};

// One work item: the stationary 128-row block `blk` of head `hx` (K/V head in the KV pass,
// query head in the Q pass) and the range [lo, hi) of streaming tiles it meets (query tiles
// in the KV pass, repeated for each of the kv_group query heads; key blocks in the Q pass).
struct BwdItem {
  int b, hx, blk, lo, hi, nsteps;  // nsteps = 0: a block past its sequence's end (packed batch)
  int s0, len, tb;  // first row of the sequence in the tensors, its length, TMA batch coordinate
};

// Item t -> work, longest first inside equal-size L2 groups of heads (see decode_item).
template <bool KV, bool WIN, bool VAR>
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
  int nblk = p.nblk;  // 128-row blocks of this item's sequence
  if (VAR) {
    const int a = min(max(__ldg(p.cu_seqlens + it.b), 0), p.total);
    const int e = min(max(__ldg(p.cu_seqlens + it.b + 1), a), p.total);
    it.s0 = a;
    it.len = min(e - a, p.N);
    it.tb = 0;
    nblk = (it.len + kBlockM - 1) / kBlockM;
  } else {
    it.s0 = 0;
    it.len = p.N;
    it.tb = it.b;
  }
  if (KV) {
    // Causal: key block blk is seen by query tiles >= blk, so low blocks are the long ones.
    it.blk = rb;
    it.lo = p.causal ? it.blk : 0;
    it.hi = nblk;
    if (WIN) it.hi = min(nblk, (it.blk * kBlockN + kBlockN - 1 + p.window) / kBlockM + 1);
    it.nsteps = p.kv_group * (it.hi - it.lo);
  } else {
    it.blk = MB - 1 - rb;
    it.lo = WIN ? max(0, it.blk * kBlockM - p.window) / kBlockN : 0;
    it.hi = p.causal ? it.blk + 1 : nblk;
    it.nsteps = it.hi - it.lo;
  }
  if (it.blk >= nblk) it.nsteps = 0;
  return it;
}

// ndelta[bh][i] = -sum_d dO[b,h,i,d] O[b,h,i,d] (fp32) and nlse2[bh][i] = -lse[bh][i] log2(e)
// for i < Npad (padding rows: ndelta 0, nlse2 -inf), stored negated so the elementwise
// warps add them with one packed instruction. kTpr = D / 8 threads per row, each reading
// one 16-byte vector of O and of dO.
template <typename T, int D, bool VAR>
__global__ void __launch_bounds__(256) attn_bwd_prep_kernel(const T* __restrict__ o,
                                                            const T* __restrict__ dout,
                                                            const float* __restrict__ lse,
                                                            float* __restrict__ nlse2,
                                                            float* __restrict__ ndelta, long long o_sb,
                                                            long long o_sh, long long o_sn,
                                                            long long d_sb, long long d_sh,
                                                            long long d_sn, int H, int N, int Npad,
                                                            long long rows, const int* cu_seqlens,
                                                            int total) {
  constexpr int kTpr = D / 8;
  const long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) / kTpr;
  const int sub = (int)(threadIdx.x % kTpr);
  const bool in_range = row < rows;  // no early exit: every lane takes part in the shuffles
  const int i = in_range ? (int)(row % Npad) : 0;
  const long long bh = in_range ? row / Npad : 0;
  const int b = (int)(bh / H);
  const int h = (int)(bh - (long long)b * H);
  // Row i of sequence b: tensor row s0 + i (packed batch) or row i of batch b.
  int len = N;
  long long s0 = 0;
  if (VAR && in_range) {
    const int a0 = min(max(__ldg(cu_seqlens + b), 0), total);
    const int e0 = min(max(__ldg(cu_seqlens + b + 1), a0), total);
    s0 = a0;
    len = min(e0 - a0, N);
  }
  const long long ob = VAR ? 0 : (long long)b * o_sb, db = VAR ? 0 : (long long)b * d_sb;
  float acc = 0.f;
  if (in_range && i < len) {
    const uint4 a = *reinterpret_cast<const uint4*>(o + ob + h * o_sh + (s0 + i) * o_sn + sub * 8);
    const uint4 g = *reinterpret_cast<const uint4*>(dout + db + h * d_sh + (s0 + i) * d_sn + sub * 8);
    const T* av = reinterpret_cast<const T*>(&a);
    const T* gv = reinterpret_cast<const T*>(&g);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc = fmaf((float)av[e], (float)gv[e], acc);
  }
#pragma unroll
  for (int w = kTpr / 2; w > 0; w >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, w);
  if (in_range && sub == 0) {
    ndelta[row] = -acc;
    // lse: [B, H, N]; packed batch: [H, total]
    const long long li = VAR ? (long long)h * total + s0 + i : bh * N + i;
    nlse2[row] = i < len ? lse[li] * -1.4426950408889634f : -INFINITY;
  }
}

// KV = true: dK, dV pass; KV = false: dQ pass. WIN: causal sliding window in use. VAR:
// packed variable-length batch.
template <int D, typename T, bool KV, bool WIN, bool VAR>
__global__ void __launch_bounds__(BwdCfg<D>::kThreads, 1)
    attn_bwd_sm100_kernel(const __grid_constant__ CUtensorMap tmX1,
                          const __grid_constant__ CUtensorMap tmX2,
                          const __grid_constant__ CUtensorMap tmY1,
                          const __grid_constant__ CUtensorMap tmY2, const BwdParams p) {
  using C = BwdCfg<D>;
  using Plan = BwdSmem<D>;
  constexpr int NS = C::kNS;
  constexpr int kEmu = D == 64 ? APEX_BWD_EMU64 : APEX_BWD_EMU128;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  if (Plan::kDynamicBytes == Plan::kBytes && (raw_addr & 1023u) != 0) {
    // The plan needs the whole 227 KB and the base is not 1 KB aligned: report, do nothing.
    if (threadIdx.x == 0) report_error(p.status, p.host_flag, kStatusSmemAlign);
    return;
  }
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
    ptx::mbar_init(bar(Plan::kXEmpty), KV ? 1 : 256);  // KV: MMA commit; Q: copied to TMEM
    ptx::mbar_init(bar(Plan::kXTFull), 256);
    ptx::mbar_init(bar(Plan::kXTFree), 1);
    ptx::mbar_init(bar(Plan::kT1Full), 1);
    ptx::mbar_init(bar(Plan::kT1Free), 256);
    for (int h = 0; h < 2; ++h) {
      ptx::mbar_init(bar(Plan::kT2Full + h), 1);
      ptx::mbar_init(bar(Plan::kT2Free + h), 1);
      ptx::mbar_init(bar(Plan::kPdSFull + h), 128);
      ptx::mbar_init(bar(Plan::kStatsFull + h), 1);
      ptx::mbar_init(bar(Plan::kStatsEmpty + h), 256);
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
  const Waiter W{abort_flag, p.status, p.timeout_ns, p.host_flag};

  if (warp < C::kWarpMma) {
    // ======================================================== elementwise ===
    ptx::setmaxnreg_inc<C::kRegsElementwise>();
    const int quarter = warp & 3;
    const int half = warp >> 2;          // column half of the 128 x 128 tile
    const int r = quarter * 32 + lane;   // row (TMEM lane)
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tT1 = tmem + lane_off + (uint32_t)(C::kT1 + 64 * half);
    const uint32_t tT2 = tmem + lane_off + (uint32_t)(C::kT2 + 64 * half);
    const float* stats = reinterpret_cast<const float*>(smem + Plan::kStats);
    const float c = p.scale_log2;
    uint32_t t1_par = 0, t2_par = 0, af_par = 0, x_par = 0, xt_par = 0;
    int items_seen = 0;
    int gstep = 0;  // steps processed by this CTA
    bool ok = true;
    ItemReader reader;
    while (ok) {
      int t;
      if (!(ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, true, t)) || t < 0) break;
      const BwdItem it = decode_bwd<KV, WIN, VAR>(t, p);
      if (it.nsteps == 0) continue;  // block past its sequence's end: no work, no barrier
      const int nq = it.hi - it.lo;
      float row_nlse2 = 0.f, row_ndelta = 0.f;
      if (!KV) {
        // Q pass: this thread's query row statistics, fixed for the item.
        const long long idx = ((long long)it.b * p.H + it.hx) * p.Npad + it.blk * kBlockM + r;
        row_nlse2 = p.nlse2[idx];
        row_ndelta = p.ndelta[idx];
        // Copy the item's Q (warpgroup 0) or dO (warpgroup 1) row r from the swizzled
        // shared-memory tile into TMEM as 16-bit pairs: the A operand of the score GEMMs.
        if (!(ok = W.wait_warp(bar(Plan::kXFull), x_par))) break;
        x_par ^= 1;
        if (items_seen > 0) {  // the previous item's last score GEMMs read the TMEM copy
          if (!(ok = W.wait_warp(bar(Plan::kXTFree), xt_par))) break;
          xt_par ^= 1;
          ptx::tc_fence_after();
        }
        const uint32_t src = sbase + (half ? Plan::kX2 : Plan::kX1) + r * 128;
        const uint32_t dst = tmem + lane_off + (uint32_t)(half ? C::kXdO : C::kXQ);
#pragma unroll
        for (int cc = 0; cc < D / 64; ++cc) {
          uint32_t x[32];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint4 q4 = ptx::ld_shared_v4(src + cc * Plan::kChunkBytes + ((u ^ (r & 7)) << 4));
            x[4 * u] = q4.x;
            x[4 * u + 1] = q4.y;
            x[4 * u + 2] = q4.z;
            x[4 * u + 3] = q4.w;
          }
          ptx::tmem_st32(dst + cc * 32, x);
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(Plan::kXTFull));
        ptx::mbar_arrive(bar(Plan::kXEmpty));  // the shared-memory tiles may be refilled
      }
      ++items_seen;
      for (int s = 0; s < it.nsteps && ok; ++s, ++gstep) {
        const int ytile = it.lo + (KV ? s % nq : s);
        // KV pass: -lse2 / -delta of this step's query tile (double-buffered by step).
        const int sslot = gstep & 1;
        const float* st_nlse = stats + sslot * 256 + 64 * half;
        const float* st_ndelta = st_nlse + 128;
        if (KV && !(ok = W.wait_warp(bar(Plan::kStatsFull + sslot), (uint32_t)(gstep >> 1) & 1u))) break;
        // Mask geometry: qi - kj = dq0 + (KV ? col - row : row - col).
        const int it_q = KV ? ytile : it.blk;
        const int jb_k = KV ? it.blk : ytile;
        const int dq0 = (it_q - jb_k) * kBlockM;
        // Packed batch, Q pass, full attention: keys past the sequence end belong to the next
        // sequence (not zero-filled) and are masked.
        const bool key_tail = VAR && !KV && !p.causal && (ytile + 1) * kBlockN > it.len;
        const bool masked = (p.causal && it_q == jb_k) || (WIN && dq0 + kBlockM - 1 > p.window) || key_tail;
        const int colbase = 64 * half;
        if (!(ok = W.wait_warp(bar(Plan::kT1Full), t1_par))) break;
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
          // S is in registers: the next score GEMM may overwrite T1.
          ptx::tc_fence_before();
          ptx::mbar_arrive(bar(Plan::kT1Free));
          if (KV) {
#pragma unroll
            for (int e = 0; e < 64; e += 4) {
              const float4 l4 = *reinterpret_cast<const float4*>(st_nlse + e);
              const float2 x0 = __ffma2_rn(make_float2(__uint_as_float(v[e >> 5][e & 31]), __uint_as_float(v[e >> 5][(e & 31) + 1])),
                                           make_float2(c, c), make_float2(l4.x, l4.y));
              const float2 x1 = __ffma2_rn(make_float2(__uint_as_float(v[e >> 5][(e & 31) + 2]), __uint_as_float(v[e >> 5][(e & 31) + 3])),
                                           make_float2(c, c), make_float2(l4.z, l4.w));
              pv[e] = x0.x;
              pv[e + 1] = x0.y;
              pv[e + 2] = x1.x;
              pv[e + 3] = x1.y;
            }
          } else {
            const float2 nl = make_float2(row_nlse2, row_nlse2);
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
            if ((p.causal && dqk < 0) || (WIN && dqk > p.window) ||
                (key_tail && ytile * kBlockN + colbase + e >= it.len))
              pv[e] = -INFINITY;
          }
        }
        if (masked || kEmu == 0) {
#pragma unroll
          for (int e = 0; e < 64; ++e) pv[e] = ptx::ex2(pv[e]);  // masked: exactly 0
        } else {
#pragma unroll
          for (int e = 0; e < 64; e += 2) {
            if (((e >> 1) & 7) < kEmu) {
              const float2 y = exp2_poly_pair(make_float2(pv[e], pv[e + 1]));
              pv[e] = y.x;
              pv[e + 1] = y.y;
            } else {
              pv[e] = ptx::ex2(pv[e]);
              pv[e + 1] = ptx::ex2(pv[e + 1]);
            }
          }
        }
        uint32_t pk_p[32];
        if (KV) {
#pragma unroll
          for (int e = 0; e < 32; ++e) pk_p[e] = DType<T>::pack(pv[2 * e], pv[2 * e + 1]);
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
          // dP is in registers; P_h goes into this warpgroup's first 32 T2 columns now, so
          // its packed registers die before dS is formed.
          if (KV) ptx::tmem_st32(tT2, pk_p);
          uint32_t pk_s[32];
          if (KV) {
#pragma unroll
            for (int e = 0; e < 64; e += 4) {  // dS = P (dP - delta), two lanes per instruction
              const float4 d4 = *reinterpret_cast<const float4*>(st_ndelta + e);
              const float2 a01 = __fmul2_rn(make_float2(pv[e], pv[e + 1]),
                                            __fadd2_rn(make_float2(__uint_as_float(v[e >> 5][e & 31]), __uint_as_float(v[e >> 5][(e & 31) + 1])),
                                                       make_float2(d4.x, d4.y)));
              const float2 a23 = __fmul2_rn(make_float2(pv[e + 2], pv[e + 3]),
                                            __fadd2_rn(make_float2(__uint_as_float(v[e >> 5][(e & 31) + 2]), __uint_as_float(v[e >> 5][(e & 31) + 3])),
                                                       make_float2(d4.z, d4.w)));
              pk_s[e >> 1] = DType<T>::pack(a01.x, a01.y);
              pk_s[(e >> 1) + 1] = DType<T>::pack(a23.x, a23.y);
            }
            ptx::tmem_st32(tT2 + 32, pk_s);  // dS_h after P_h
            ptx::mbar_arrive(bar(Plan::kStatsEmpty + sslot));  // statistics read
          } else {
            const float2 nd = make_float2(row_ndelta, row_ndelta);
#pragma unroll
            for (int e = 0; e < 64; e += 2) {
              const float2 a = __fmul2_rn(make_float2(pv[e], pv[e + 1]),
                                          __fadd2_rn(make_float2(__uint_as_float(v[e >> 5][e & 31]), __uint_as_float(v[e >> 5][(e & 31) + 1])), nd));
              pk_s[e >> 1] = DType<T>::pack(a.x, a.y);
            }
            ptx::tmem_st32(tT2, pk_s);
          }
          ptx::tmem_wait_st();
        }
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(Plan::kPdSFull + half));
      }
      if (!ok) break;
      // ---- epilogue: Acc1 * scale -> out1 (dK | dQ), Acc2 -> out2 (dV) ----
      if (!(ok = W.wait_warp(bar(Plan::kAccFull), af_par))) break;
      af_par ^= 1;
      ptx::tc_fence_after();
      const int row = it.blk * kBlockM + r;
      const bool valid = row < it.len;
      constexpr int kHalfCols = D / 2;
      auto store = [&](void* base, long long sb, long long sh, long long sn, int acc_col, float scale) {
        T* dst = reinterpret_cast<T*>(base) + (VAR ? 0LL : (long long)it.b * sb) + (long long)it.hx * sh +
                 (long long)(it.s0 + row) * sn + half * kHalfCols;
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
    ptx::setmaxnreg_dec<C::kRegsOther>();
    // ================================================================ MMA ===
    // Issue order, software-pipelined across steps (s = step, all 128 x 128 tiles):
    //   G1(s)      T1 = X1 Y1(s)^T          after the elementwise warps read S(s-1)
    //   A(s-1)     accumulating GEMMs of the previous step (as its P / dS halves arrive):
    //              KV: dV += P^T dO, dK += dS^T Q;  Q pass: dQ += dS K
    //   G2(s)      T2 = X2 Y2(s)^T          after A(s-1) completed (it reads T2)
    // so the score GEMM of step s runs while the elementwise warps work on step s-1.
    constexpr uint32_t idNT = make_idesc<T>(kBlockM, kBlockN, false);  // T1 = X Y^T
    constexpr uint32_t idNT64 = make_idesc<T>(kBlockM, 64, false);     // T2_h = X Y_h^T
    constexpr uint32_t idAcc = make_idesc<T>(kBlockM, D, true);        // Acc += A_h(TMEM) Y_h
    constexpr uint32_t kHalfRows = 64 * 128;  // byte offset of row 64 inside a 128-row chunk
    // dP as two 64-column GEMMs. Free in the Q pass (A = dO from TMEM, B 2 KB per
    // instruction); in the KV pass both operands come from shared memory and a 64-wide
    // instruction reads 6 KB in 32 tensor cycles (it runs at 48).
    constexpr bool kSplitDP = !KV || APEX_BWD_SPLIT_DP_KV;
    const uint32_t sX1 = sbase + Plan::kX1;
    const uint32_t sX2 = sbase + Plan::kX2;
    const uint32_t sRing = sbase + Plan::kRing;
    // T = X Y^T over D (Y: 128 rows, or 64 from sB with idesc idNT64): X from shared memory
    // (KV pass) or from TMEM (Q pass, x_tmem).
    auto gemm_nt = [&](uint32_t d_tmem, uint32_t sA, uint32_t x_tmem, uint32_t sB, uint32_t idesc) {
      const uint64_t a0 = make_sdesc_sw128(sA, 16, 1024);
      const uint64_t b0 = make_sdesc_sw128(sB, 16, 1024);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (uint32_t)((kk >> 2) * Plan::kChunkBytes + (kk & 3) * 32) >> 4;
        if (KV) ptx::umma_ss_warp(d_tmem, a0 + off, b0 + off, idesc, kk > 0 ? 1u : 0u);
        else ptx::umma_ts_warp(d_tmem, x_tmem + (uint32_t)(8 * kk), b0 + off, idesc, kk > 0 ? 1u : 0u);
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
    const uint32_t tT1 = tmem + C::kT1, tT2 = tmem + C::kT2;
    const uint32_t tAcc1 = tmem + C::kAcc1, tAcc2 = tmem + C::kAcc2;
    Ring<NS> ring;
    uint32_t x_par = 0, t1f_par = 0, t2f_par = 0, pds_par = 0, ae_par = 0;  // bit h: half h
    int steps_issued = 0, items_accumulated = 0;
    bool ok = true;
    struct Pending {
      bool valid;
      int st1, st2;
      bool first, last;  // first / last step of its item
    };
    Pending pend{false, 0, 0, false, false};
    auto acquire = [&]() -> int {
      const int st = ring.stage;
      const uint32_t ph = ring.phase;
      ring.next();
      if (!W.wait_warp(bar(Plan::kRingFull + st), ph)) return -1;
      ptx::tc_fence_after();
      return st;
    };
    // A(step): accumulating GEMMs of a step whose G1, G2 were issued earlier.
    auto accumulate = [&](const Pending& pd) -> bool {
      if (pd.first && items_accumulated > 0) {  // the epilogue must have drained the accumulators
        if (!W.wait_warp(bar(Plan::kAccEmpty), ae_par)) return false;
        ae_par ^= 1;
        ptx::tc_fence_after();
      }
      const uint32_t sY1 = sRing + pd.st1 * Plan::kTileBytes;
      const uint32_t sY2 = sRing + pd.st2 * Plan::kTileBytes;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        if (!W.wait_warp(bar(Plan::kPdSFull + h), (pds_par >> h) & 1u)) return false;
        pds_par ^= 1u << h;
        ptx::tc_fence_after();
        const bool acc = !pd.first || h > 0;
        const uint32_t tP = tT2 + (uint32_t)(64 * h);
        if (KV) {
          gemm_acc(tAcc2, tP, sY2 + h * kHalfRows, acc);       // dV += P_h^T dO_h
          gemm_acc(tAcc1, tP + 32, sY1 + h * kHalfRows, acc);  // dK += dS_h^T Q_h
        } else {
          gemm_acc(tAcc1, tP, sY1 + h * kHalfRows, acc);       // dQ += dS_h K_h
        }
        ptx::tc_commit_warp(bar(Plan::kT2Free + h));
      }
      ptx::tc_commit_warp(bar(Plan::kRingEmpty + pd.st1));
      if (KV) ptx::tc_commit_warp(bar(Plan::kRingEmpty + pd.st2));
      if (pd.last) {
        ptx::tc_commit_warp(bar(Plan::kAccFull));
        ++items_accumulated;
      }
      return true;
    };
    ItemReader reader;
    while (ok) {
      int t;
      if (!(ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, true, t)) || t < 0) break;
      const BwdItem it = decode_bwd<KV, WIN, VAR>(t, p);
      if (it.nsteps == 0) continue;  // block past its sequence's end
      // Q pass: the elementwise warps copy the next item's X only after finishing this
      // item's epilogue, which waits for the last A(); issue it before waiting for X.
      if (!KV && pend.valid) {
        if (!(ok = accumulate(pend))) break;
        pend.valid = false;
      }
      if (!(ok = W.wait_warp(bar(KV ? Plan::kXFull : Plan::kXTFull), x_par))) break;
      x_par ^= 1;
      ptx::tc_fence_after();
      for (int s = 0; s < it.nsteps && ok; ++s) {
        const int st1 = acquire();
        ok = st1 >= 0;
        if (!ok) break;
        if (steps_issued > 0) {  // the elementwise warps hold S(s-1) in registers
          if (!(ok = W.wait_warp(bar(Plan::kT1Free), t1f_par))) break;
          t1f_par ^= 1;
          ptx::tc_fence_after();
        }
        gemm_nt(tT1, sX1, tmem + C::kXQ, sRing + st1 * Plan::kTileBytes, idNT);
        ptx::tc_commit_warp(bar(Plan::kT1Full));
        if (pend.valid) {
          if (!(ok = accumulate(pend))) break;
          pend.valid = false;
        }
        const int st2 = acquire();
        ok = st2 >= 0;
        if (!ok) break;
        if (kSplitDP) {
          // dP in two column halves: half h of T2 is rewritten as soon as A_h(s-1) finished
          // reading P_h / dS_h from it, and elementwise warpgroup h starts on it at once.
#pragma unroll 1
          for (int h = 0; h < 2 && ok; ++h) {
            if (steps_issued > 0) {
              if (!(ok = W.wait_warp(bar(Plan::kT2Free + h), (t2f_par >> h) & 1u))) break;
              t2f_par ^= 1u << h;
              ptx::tc_fence_after();
            }
            gemm_nt(tT2 + (uint32_t)(64 * h), sX2, tmem + C::kXdO,
                    sRing + st2 * Plan::kTileBytes + h * kHalfRows, idNT64);
            ptx::tc_commit_warp(bar(Plan::kT2Full + h));
          }
          if (!ok) break;
        } else {
          if (steps_issued > 0) {
#pragma unroll 1
            for (int h = 0; h < 2 && ok; ++h) {
              ok = W.wait_warp(bar(Plan::kT2Free + h), (t2f_par >> h) & 1u);
              t2f_par ^= 1u << h;
            }
            if (!ok) break;
            ptx::tc_fence_after();
          }
          gemm_nt(tT2, sX2, tmem + C::kXdO, sRing + st2 * Plan::kTileBytes, idNT);
          ptx::tc_commit_warp(bar(Plan::kT2Full));
          ptx::tc_commit_warp(bar(Plan::kT2Full + 1));
        }
        if (!KV) ptx::tc_commit_warp(bar(Plan::kRingEmpty + st2));  // V: only dP reads it
        if (s == it.nsteps - 1) ptx::tc_commit_warp(bar(KV ? Plan::kXEmpty : Plan::kXTFree));  // last reads of X
        pend = Pending{true, st1, st2, s == 0, s == it.nsteps - 1};
        ++steps_issued;
      }
    }
    if (ok && pend.valid) ok = accumulate(pend);
    ptx::tc_commit_warp(bar(Plan::kDrain));
    if (lane == 0) drain_wait(bar(Plan::kDrain), 0, p.timeout_ns, p.status, p.host_flag);
    __syncwarp();
  } else {
    ptx::setmaxnreg_dec<C::kRegsOther>();
    // ============================================== scheduler + producer ===
    if (warp == C::kWarpProd && lane == 0) {
      const uint64_t pol_x = ptx::policy_evict_first();  // read by this item only
      const uint64_t pol_y = ptx::policy_evict_last();   // re-read by every block of the head
      const uint32_t sX1 = sbase + Plan::kX1;
      const uint32_t sX2 = sbase + Plan::kX2;
      const uint32_t sRing = sbase + Plan::kRing;
      const uint32_t sStats = sbase + Plan::kStats;
      Ring<NS> ring;
      uint32_t xe_par = 1;
      int fills = 0, x_fills = 0, stat_fills = 0;
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
        const BwdItem it = decode_bwd<KV, WIN, VAR>(t, p);
        if (it.nsteps == 0) continue;  // block past its sequence's end
        if (!(ok = W.wait(bar(Plan::kXEmpty), xe_par))) break;
        xe_par ^= 1;
        ptx::mbar_arrive_expect_tx(bar(Plan::kXFull), 2u * Plan::kTileBytes);
        load_tile(sX1, &tmX1, bar(Plan::kXFull), it.s0 + it.blk * kBlockM, it.hx, it.tb, pol_x);
        load_tile(sX2, &tmX2, bar(Plan::kXFull), it.s0 + it.blk * kBlockM, it.hx, it.tb, pol_x);
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
            ptx::mbar_arrive_expect_tx(bar(Plan::kRingFull + st), (uint32_t)Plan::kTileBytes);
            load_tile(sRing + st * Plan::kTileBytes, k == 0 ? &tmY1 : &tmY2, bar(Plan::kRingFull + st),
                      it.s0 + ytile * kBlockN, hy, it.tb, pol_y);
            ++fills;
          }
          if (KV && ok) {
            // lse2 / delta of the query tile into stats slot (step & 1), after the
            // elementwise warps released it (two steps back).
            const int sslot = stat_fills & 1;
            if (!(ok = W.wait(bar(Plan::kStatsEmpty + sslot), ((uint32_t)(stat_fills >> 1) & 1u) ^ 1u))) break;
            const long long idx = ((long long)it.b * p.H + hy) * p.Npad + (long long)ytile * kBlockM;
            ptx::mbar_arrive_expect_tx(bar(Plan::kStatsFull + sslot), 1024u);
            ptx::bulk_load(sStats + sslot * Plan::kStatsBytes, p.nlse2 + idx, 512u, bar(Plan::kStatsFull + sslot), pol_y);
            ptx::bulk_load(sStats + sslot * Plan::kStatsBytes + 512, p.ndelta + idx, 512u, bar(Plan::kStatsFull + sslot), pol_y);
            ++stat_fills;
          }
        }
      }
      // Let every load this thread issued land before the CTA exits.
      const int last = fills < NS ? fills : NS;
      for (int k = 0; k < last; ++k) {
        const int f = fills - 1 - k;
        drain_wait(bar(Plan::kRingFull + (f % NS)), (uint32_t)((f / NS) & 1), p.timeout_ns, p.status, p.host_flag);
      }
      if (x_fills > 0) drain_wait(bar(Plan::kXFull), (uint32_t)((x_fills - 1) & 1), p.timeout_ns, p.status, p.host_flag);
      for (int k = stat_fills > 2 ? stat_fills - 2 : 0; k < stat_fills; ++k)
        drain_wait(bar(Plan::kStatsFull + (k & 1)), (uint32_t)(k >> 1) & 1u, p.timeout_ns, p.status, p.host_flag);
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
