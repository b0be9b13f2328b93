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
// The fused mode (DQ = true) instead runs launch 2 with a fifth GEMM per step, dQ = dS K,
// whose tiles warps 12-15 add into a zeroed fp32 accumulator with TMA reduce-adds (staged
// through shared memory); a cast kernel (attn_bwd_dq_cast_kernel) then writes
// dq = scale * acc.
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
// warps 10-11 only give their registers to the elementwise warpgroups. The fused form adds
// the dQ warps 12-15 (512 threads). APEX_BWD_WG4 (off) runs four elementwise warpgroups of
// 32 columns instead (640 threads; MMA warp 16, producer warp 17).
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
// Four elementwise warpgroups in the two-pass backward (see BwdCfg::kWG), with this many
// registers each (the MMA/producer warpgroup gets 480 - 4 x this; 640 threads x 96). Off:
// all backward tests pass with it, but it measured level (C2 0.598 vs 0.604-0.609 ms, C3
// 6.24-6.27 vs 6.09-6.21 ms): the elementwise latency is not what paces the passes.
#ifndef APEX_BWD_WG4
#define APEX_BWD_WG4 0
#endif
#ifndef APEX_BWD_WG4_REGS
#define APEX_BWD_WG4_REGS 104
#endif
#ifndef APEX_BWD_T2X2
#define APEX_BWD_T2X2 0
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
  // Fused form: fp32 dQ accumulator, zeroed before the launch; [B][H][N][D], or [H][total][D]
  // for a packed batch. Unscaled: it holds dS K, and the cast to the output applies scale.
  float* dq_acc;
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

// DQ: the fused one-pass form of the dK/dV pass (see attn_bwd_sm100_kernel).
template <int D, bool DQ = false>
struct BwdCfg {
  static_assert(D == 64 || D == 128, "backward head dims 64, 128");
  // Streaming ring stages (one 128-row tile each). A stage frees when the accumulating GEMMs
  // of its step finish and takes ~1300 cycles to refill from L2, so the ring holds about
  // two and a half steps (two tiles per step). The fused form gives 64 KB to the dS tile
  // and the dQ staging chunks.
  static constexpr int kNS = DQ ? (D == 64 ? 8 : 3) : (D == 64 ? 10 : 5);
  // Elementwise warpgroups. Warpgroup w takes the tile's columns [kCols w, kCols (w + 1))
  // for every row (thread = TMEM lane = row). The two-pass form runs four (32 columns
  // each), so four elementwise warps share each SM sub-partition and hide each other's
  // TMEM-load and math latency (the elementwise work is latency-bound: ~30 % issue with
  // two). The fused form keeps two: its dQ warpgroup leaves no register room for four.
  static constexpr int kWG = APEX_BWD_WG4 && !DQ ? 4 : 2;
  static constexpr int kCols = 128 / kWG;
  // Warps: the elementwise warpgroups, then MMA, producer, idle warps (+ 4 dQ warps in the
  // fused form). Registers are granted per warpgroup, so the launch budget is kThreads x
  // (65536 / kThreads); setmaxnreg moves it to the elementwise warpgroups (the split must
  // not exceed the launch allocation, or setmaxnreg.inc would never return).
  static constexpr int kThreads = 128 * (kWG + 1) + (DQ ? 128 : 0);
  static constexpr int kWarpMma = 4 * kWG;
  static constexpr int kWarpProd = kWarpMma + 1;
  static constexpr int kWarpDq = kWarpMma + 4;  // fused form: 4 warps reduce dQ tiles into global memory
  // Fused splits: the ones without spills in the plain (unwindowed, batched) builds.
  static constexpr int kRegsElementwise = kWG == 4 ? APEX_BWD_WG4_REGS : (DQ ? 200 : 224);
  static constexpr int kRegsOther = kWG == 4 ? 480 - 4 * APEX_BWD_WG4_REGS : (DQ && D == 64 ? 48 : 56);
  static constexpr int kRegsDq = DQ ? (D == 64 ? 64 : 56) : 0;
  static constexpr int kLaunchRegs = (65536 / kThreads) / 8 * 8;
  static_assert(128 * (kWG * kRegsElementwise + kRegsOther + kRegsDq) <= kThreads * kLaunchRegs,
                "setmaxnreg split exceeds the launch register allocation");
  // TMEM columns: T1 scores, T2 dP (then packed P / dS), Acc1 dK | dQ, Acc2 dV (KV pass),
  // XQ / XdO the item's Q and dO as 16-bit pairs (Q pass).
  static constexpr int kT1 = 0;
  static constexpr int kT2 = 128;
  static constexpr int kAcc1 = 256;
  static constexpr int kAcc2 = 256 + D;
  static constexpr int kXQ = 256 + D;
  static constexpr int kXdO = kXQ + D / 2;
  // Two-pass form at d = 64 (APEX_BWD_T2X2): a second T2 buffer in the 128 free columns
  // [384, 512), used by odd steps, so the dP GEMM of step s waits only for the accumulating
  // GEMMs of step s - 2. Off: all backward tests pass with it, but C2 measured 3 % slower
  // (0.623 vs 0.603 ms): the P / dS hand-off through T2 is not what paces the passes.
  static constexpr int kT2Bufs = D == 64 && !DQ && APEX_BWD_T2X2 ? 2 : 1;
  static constexpr int kT2b = 384;
  static __host__ __device__ constexpr int t2_col(int b) { return b == 0 ? kT2 : kT2b; }
  // Fused form: the step's dQ tile (fp32, 128 query rows x D). At d = 64 two buffers fit
  // behind dV. At d = 128 TMEM is full: dQ borrows T2 once the step's dV and dK GEMMs have
  // read P and dS from it, and the next dP GEMM writes each 64-column half of T2 once the
  // dQ warps have read that half out. T1 stays free for the next score GEMM, which keeps
  // running during the elementwise work.
  static constexpr int kDqBufs = D == 64 ? 2 : 1;
  static constexpr int kDq = D == 64 ? 256 + 2 * D : kT2;
  static constexpr bool kDqInT2 = DQ && D == 128;
  static constexpr int kDqStage = 2;  // 16 KB shared-memory staging chunks (128 rows x 32 fp32);
                                      // the dQ warps' bulk_wait_group_read1 assumes 2
  static_assert(kAcc2 + D <= 512 && kXdO + D / 2 <= 512, "TMEM plan overflows 512 columns");
  static_assert(!DQ || kDqInT2 || kDq + kDqBufs * D <= 512, "dQ buffers overflow TMEM");
  static_assert(kT2Bufs == 1 || (kAcc2 + D <= kT2b && kXdO + D / 2 <= kT2b), "second T2 buffer overlaps");
};

template <int D, bool DQ = false>
struct BwdSmem {
  using C = BwdCfg<D, DQ>;
  static constexpr int NS = C::kNS;
  static constexpr int kChunkBytes = kBlockM * 128;
  static constexpr int kTileBytes = kBlockM * D * 2;
  static constexpr int kX1 = 0;
  static constexpr int kX2 = kX1 + kTileBytes;
  static constexpr int kRing = kX2 + kTileBytes;
  // Fused form: dS^T of the step, 128 key rows x 128 query columns (16-bit) in two SW128
  // chunks of 64 queries; the dQ GEMM reads it as an MN-major A operand (dS).
  static constexpr int kDs = kRing + NS * kTileBytes;
  static constexpr int kDsBytes = DQ ? 2 * kChunkBytes : 0;
  // Fused form: staging chunks of the dQ tile for the TMA reduce, each 128 rows x 32 fp32
  // (128 bytes per row, 128-byte swizzle: the box layout of the accumulator's tensor map).
  static constexpr int kStage = kDs + kDsBytes;
  static constexpr int kStageBytes = DQ ? C::kDqStage * kChunkBytes : 0;
  // KV pass: per-column statistics of the step's query tile, double-buffered:
  // float [2][256] = -lse2[128], -delta[128].
  static constexpr int kStats = kStage + kStageBytes;
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
  // [T2 buffer b][half h] at index 2 b + h:
  static constexpr int kT2Full = kT1Free + 1;   // [4] dP of column half h
  static constexpr int kT2Free = kT2Full + 4;   // [4] accumulating GEMMs of half h done
  static constexpr int kPdSFull = kT2Free + 4;  // [4] P_h / dS_h packed in T2
  static constexpr int kStatsFull = kPdSFull + 4;    // [2]
  static constexpr int kStatsEmpty = kStatsFull + 2;  // [2]
  static constexpr int kAccFull = kStatsEmpty + 2;
  static constexpr int kAccEmpty = kAccFull + 1;
  static constexpr int kDrain = kAccEmpty + 1;
  static constexpr int kDqFull = kDrain + 1;    // [2] fused form: dQ tile in TMEM buffer b
  // [2] fused form: dQ buffer b read out (d = 128: 64-column half b of the one buffer)
  static constexpr int kDqFree = kDqFull + 2;
  static constexpr int kDsFree = kDqFree + 2;   // fused form, d = 64: the dQ GEMM read the dS tile
  static constexpr int kItemFull = kDsFree + 1;
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
  static_assert(kDs % 1024 == 0, "SW128 tiles need 1 KB alignment");
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

// Fused backward, last launch: dq = scale * acc in the output dtype, for the rows the
// two-pass form writes: row i < len of every (batch, head). Rows are walked as in the prep
// kernel, [B * H][Npad]; acc is fp32 [B][H][N][D], or [H][total][D] for a packed batch
// (sequence b at token cu_seqlens[b], clamped as in the attention kernels). kTpr = D / 8
// threads per row, each converting 8 elements.
template <typename T, int D, bool VAR>
__global__ void __launch_bounds__(256) attn_bwd_dq_cast_kernel(const float* __restrict__ acc, T* __restrict__ dq,
                                                               long long sb, long long sh, long long sn, int H,
                                                               int N, int Npad, long long rows,
                                                               const int* cu_seqlens, int total, float scale) {
  constexpr int kTpr = D / 8;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long row = idx / kTpr;
  if (row >= rows) return;
  const int sub = (int)(idx % kTpr);
  const int i = (int)(row % Npad);
  const long long bh = row / Npad;
  const int b = (int)(bh / H);
  const int h = (int)(bh - (long long)b * H);
  long long arow, orow;  // accumulator row, and element offset of the output row
  if (VAR) {
    const int a0 = min(max(__ldg(cu_seqlens + b), 0), total);
    const int e0 = min(max(__ldg(cu_seqlens + b + 1), a0), total);
    if (i >= min(e0 - a0, N)) return;
    arow = (long long)h * total + a0 + i;
    orow = (long long)h * sh + (long long)(a0 + i) * sn;
  } else {
    if (i >= N) return;
    arow = bh * N + i;
    orow = (long long)b * sb + (long long)h * sh + (long long)i * sn;
  }
  const float4* src = reinterpret_cast<const float4*>(acc + arow * D + sub * 8);
  const float4 x = src[0], y = src[1];
  uint4 o;
  o.x = DType<T>::pack(x.x * scale, x.y * scale);
  o.y = DType<T>::pack(x.z * scale, x.w * scale);
  o.z = DType<T>::pack(y.x * scale, y.y * scale);
  o.w = DType<T>::pack(y.z * scale, y.w * scale);
  *reinterpret_cast<uint4*>(dq + orow + sub * 8) = o;
}

// KV = true: dK, dV pass; KV = false: dQ pass. WIN: causal sliding window in use. VAR:
// packed variable-length batch. DQ (with KV): the fused one-pass backward. Each step also
// writes dS^T to shared memory and computes the step's dQ tile, dQ(query tile) = dS K
// (A = the dS^T tile read MN-major, B = the item's K read MN-major), into TMEM; warps 12-15
// read it out through shared-memory staging chunks and add it into the fp32 accumulator
// p.dq_acc with TMA reduce-adds over tmDq (fp32 (D, rows, B * H), or (D, total, H) for a
// packed batch; box 32 x 128 x 1). Five GEMMs per step instead of the seven of the two
// passes; dQ sums in whatever order the CTAs reach it, so it is not bitwise reproducible.
template <int D, typename T, bool KV, bool WIN, bool VAR, bool DQ = false>
__global__ void __launch_bounds__(BwdCfg<D, DQ>::kThreads, 1)
    attn_bwd_sm100_kernel(const __grid_constant__ CUtensorMap tmX1,
                          const __grid_constant__ CUtensorMap tmX2,
                          const __grid_constant__ CUtensorMap tmY1,
                          const __grid_constant__ CUtensorMap tmY2,
                          const __grid_constant__ CUtensorMap tmDq, const BwdParams p) {
  static_assert(!DQ || KV, "the fused form is a variant of the dK/dV pass");
  using C = BwdCfg<D, DQ>;
  using Plan = BwdSmem<D, DQ>;
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
    ptx::mbar_init(bar(Plan::kT1Free), 128 * C::kWG);
    for (int h = 0; h < 4; ++h) {
      ptx::mbar_init(bar(Plan::kT2Full + h), 1);
      ptx::mbar_init(bar(Plan::kT2Free + h), 1);
      ptx::mbar_init(bar(Plan::kPdSFull + h), 128 * (C::kWG / 2));  // the warpgroups of half h & 1
    }
    for (int h = 0; h < 2; ++h) {
      ptx::mbar_init(bar(Plan::kStatsFull + h), 1);
      ptx::mbar_init(bar(Plan::kStatsEmpty + h), 128 * C::kWG);
    }
    ptx::mbar_init(bar(Plan::kAccFull), 1);
    ptx::mbar_init(bar(Plan::kAccEmpty), 128 * C::kWG);
    ptx::mbar_init(bar(Plan::kDrain), 1);
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar(Plan::kDqFull + b), 1);
      ptx::mbar_init(bar(Plan::kDqFree + b), 128);
    }
    ptx::mbar_init(bar(Plan::kDsFree), 1);
    // Item-ring readers: the elementwise warps, the MMA warp (and the 4 dQ warps).
    for (int k = 0; k < kItemRing; ++k) {
      ptx::mbar_init(bar(Plan::kItemFull + k), 1);
      ptx::mbar_init(bar(Plan::kItemEmpty + k), 4 * C::kWG + 1 + (DQ ? 4 : 0));
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
    if (DQ) ptx::prefetch_tmap(&tmDq);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const Waiter W{abort_flag, p.status, p.timeout_ns, p.host_flag};

  if (warp < C::kWarpMma) {
    // ======================================================== elementwise ===
    ptx::setmaxnreg_inc<C::kRegsElementwise>();
    constexpr int kCols = C::kCols;      // tile columns of this warpgroup
    const int quarter = warp & 3;
    const int wg = warp >> 2;            // elementwise warpgroup: columns [kCols wg, kCols (wg + 1))
    const int half = wg / (C::kWG / 2);  // column half of the 128 x 128 tile
    const int r = quarter * 32 + lane;   // row (TMEM lane)
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    // T2: this warpgroup's kCols columns of dP, then its packed P (KV pass) and dS in place.
    const uint32_t tT1 = tmem + lane_off + (uint32_t)(C::kT1 + kCols * wg);
    const uint32_t tT2_0 = tmem + lane_off + (uint32_t)(C::t2_col(0) + kCols * wg);
    const uint32_t tT2_1 = tmem + lane_off + (uint32_t)(C::t2_col(1) + kCols * wg);
    const float* stats = reinterpret_cast<const float*>(smem + Plan::kStats);
    const float c = p.scale_log2;
    uint32_t t1_par = 0, af_par = 0, x_par = 0, xt_par = 0;
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
        if (wg < 2) {
        if (!(ok = W.wait_warp(bar(Plan::kXFull), x_par))) break;
        x_par ^= 1;
        if (items_seen > 0) {  // the previous item's last score GEMMs read the TMEM copy
          if (!(ok = W.wait_warp(bar(Plan::kXTFree), xt_par))) break;
          xt_par ^= 1;
          ptx::tc_fence_after();
        }
        const uint32_t src = sbase + (wg ? Plan::kX2 : Plan::kX1) + r * 128;
        const uint32_t dst = tmem + lane_off + (uint32_t)(wg ? C::kXdO : C::kXQ);
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
      }
      ++items_seen;
      for (int s = 0; s < it.nsteps && ok; ++s, ++gstep) {
        const int ytile = it.lo + (KV ? s % nq : s);
        // KV pass: -lse2 / -delta of this step's query tile (double-buffered by step).
        const int sslot = gstep & 1;
        const float* st_nlse = stats + sslot * 256 + kCols * wg;
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
        const int colbase = kCols * wg;
        if (!(ok = W.wait_warp(bar(Plan::kT1Full), t1_par))) break;
        t1_par ^= 1;
        ptx::tc_fence_after();
        float pv[kCols];
        {
          uint32_t v[kCols / 32][32];
#pragma unroll
          for (int ch = 0; ch < kCols / 32; ++ch) ptx::tmem_ld32(tT1 + 32 * ch, v[ch]);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int ch = 0; ch < kCols / 32; ++ch) ptx::reg_fence32(v[ch]);
          // S is in registers: the next score GEMM may overwrite T1.
          ptx::tc_fence_before();
          ptx::mbar_arrive(bar(Plan::kT1Free));
          if (KV) {
#pragma unroll
            for (int e = 0; e < kCols; e += 4) {
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
            for (int e = 0; e < kCols; e += 2) {
              const float2 x = __ffma2_rn(make_float2(__uint_as_float(v[e >> 5][e & 31]), __uint_as_float(v[e >> 5][(e & 31) + 1])),
                                          make_float2(c, c), nl);
              pv[e] = x.x;
              pv[e + 1] = x.y;
            }
          }
        }
        if (masked) {
#pragma unroll
          for (int e = 0; e < kCols; ++e) {
            const int dqk = dq0 + (KV ? colbase + e - r : r - colbase - e);
            if ((p.causal && dqk < 0) || (WIN && dqk > p.window) ||
                (key_tail && ytile * kBlockN + colbase + e >= it.len))
              pv[e] = -INFINITY;
          }
        }
        if (masked || kEmu == 0) {
#pragma unroll
          for (int e = 0; e < kCols; ++e) pv[e] = ptx::ex2(pv[e]);  // masked: exactly 0
        } else {
#pragma unroll
          for (int e = 0; e < kCols; e += 2) {
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
        // Fused form, packed batch, full attention: keys of this item past the sequence end
        // (the next sequence's) would add to dQ = dS K, so their rows of P (and so dS) are
        // zeroed. Their dK, dV rows are never stored. (Batched inputs read zero-filled K
        // there, and causal masks hide such keys.)
        if (DQ && VAR && !p.causal && it.blk * kBlockN + r >= it.len) {
#pragma unroll
          for (int e = 0; e < kCols; ++e) pv[e] = 0.f;
        }
        // kCols / 2 packed 16-bit pairs into this warpgroup's T2 columns.
        auto st_packed = [&](uint32_t taddr, uint32_t (&w)[kCols / 2]) {
          if constexpr (kCols == 64) ptx::tmem_st32(taddr, w);
          else ptx::tmem_st16(taddr, w);
        };
        uint32_t pk_p[kCols / 2];
        if (KV) {
#pragma unroll
          for (int e = 0; e < kCols / 2; ++e) pk_p[e] = DType<T>::pack(pv[2 * e], pv[2 * e + 1]);
        }
        // T2 buffer of this step, and the parity of its use.
        const int t2b = C::kT2Bufs == 2 ? (gstep & 1) : 0;
        const uint32_t t2u = (uint32_t)(gstep / C::kT2Bufs) & 1u;
        const uint32_t tT2 = t2b ? tT2_1 : tT2_0;
        if (!(ok = W.wait_warp(bar(Plan::kT2Full + 2 * t2b + half), t2u))) break;
        ptx::tc_fence_after();
        {
          uint32_t v[kCols / 32][32];
#pragma unroll
          for (int ch = 0; ch < kCols / 32; ++ch) ptx::tmem_ld32(tT2 + 32 * ch, v[ch]);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int ch = 0; ch < kCols / 32; ++ch) ptx::reg_fence32(v[ch]);
          // dP is in registers; P goes into this warpgroup's first kCols / 2 T2 columns
          // now, so its packed registers die before dS is formed.
          if (KV) st_packed(tT2, pk_p);
          uint32_t pk_s[kCols / 2];
          if (KV) {
#pragma unroll
            for (int e = 0; e < kCols; e += 4) {  // dS = P (dP - delta), two lanes per instruction
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
            st_packed(tT2 + kCols / 2, pk_s);  // dS after P
            if (DQ) {
              // At d = 64 the previous step's dQ GEMM may still be reading the dS tile (it is
              // issued after this step's dP GEMM); at d = 128 it completed before dP (T2).
              if (!C::kDqInT2 && gstep > 0 && !(ok = W.wait_warp(bar(Plan::kDsFree), (uint32_t)(gstep - 1) & 1u)))
                break;
              // The same dS^T row into the shared-memory tile of the dQ GEMM: chunk
              // colbase / 64 (64 queries each), row r, 16-byte unit u at position u ^ (r & 7).
              const uint32_t drow = sbase + Plan::kDs + (uint32_t)(colbase / 64) * Plan::kChunkBytes + r * 128;
              const uint32_t ub = (uint32_t)(colbase % 64) / 8;
#pragma unroll
              for (int u = 0; u < kCols / 8; ++u)
                ptx::st_shared_v4(drow + (((ub + (uint32_t)u) ^ (uint32_t)(r & 7)) << 4), pk_s[4 * u], pk_s[4 * u + 1],
                                  pk_s[4 * u + 2], pk_s[4 * u + 3]);
            }
            ptx::mbar_arrive(bar(Plan::kStatsEmpty + sslot));  // statistics read
          } else {
            const float2 nd = make_float2(row_ndelta, row_ndelta);
#pragma unroll
            for (int e = 0; e < kCols; e += 2) {
              const float2 a = __fmul2_rn(make_float2(pv[e], pv[e + 1]),
                                          __fadd2_rn(make_float2(__uint_as_float(v[e >> 5][e & 31]), __uint_as_float(v[e >> 5][(e & 31) + 1])), nd));
              pk_s[e >> 1] = DType<T>::pack(a.x, a.y);
            }
            st_packed(tT2, pk_s);
          }
          ptx::tmem_wait_st();
        }
        if (DQ) ptx::fence_proxy_async_smem();  // the dS tile, for the dQ GEMM
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(Plan::kPdSFull + 2 * t2b + half));
      }
      if (!ok) break;
      // ---- epilogue: Acc1 * scale -> out1 (dK | dQ), Acc2 -> out2 (dV) ----
      if (!(ok = W.wait_warp(bar(Plan::kAccFull), af_par))) break;
      af_par ^= 1;
      ptx::tc_fence_after();
      const int row = it.blk * kBlockM + r;
      const bool valid = row < it.len;
      constexpr int kHalfCols = D / 2;
      // Half `hh` of the columns of one accumulator. Two warpgroups: warpgroup h stores half
      // h of each; four: warpgroups 0, 1 the halves of Acc1, warpgroups 2, 3 those of Acc2.
      auto store = [&](void* base, long long sb, long long sh, long long sn, int acc_col, float scale, int hh) {
        T* dst = reinterpret_cast<T*>(base) + (VAR ? 0LL : (long long)it.b * sb) + (long long)it.hx * sh +
                 (long long)(it.s0 + row) * sn + hh * kHalfCols;
#pragma unroll 1
        for (int ch = 0; ch < kHalfCols / 32; ++ch) {
          uint32_t v[32];
          ptx::tmem_ld32(tmem + lane_off + (uint32_t)(acc_col + hh * kHalfCols + ch * 32), v);
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
      if (C::kWG == 2) {
        store(p.out1, p.o1_sb, p.o1_sh, p.o1_sn, C::kAcc1, p.out1_scale, wg);
        if (KV) store(p.out2, p.o2_sb, p.o2_sh, p.o2_sn, C::kAcc2, 1.f, wg);
      } else if (wg < 2) {
        store(p.out1, p.o1_sb, p.o1_sh, p.o1_sn, C::kAcc1, p.out1_scale, wg);
      } else if (KV) {
        store(p.out2, p.o2_sb, p.o2_sh, p.o2_sn, C::kAcc2, 1.f, wg - 2);
      }
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
    constexpr uint32_t idDq = make_idesc<T>(kBlockM, D, true, true);   // dQ = dS K, both MN-major
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
    // A: 128 x 64 16-bit operand packed in TMEM from a_tmem: 8 columns per 16 of its K
    // (the tile's columns); B: 64 rows x D. With two elementwise warpgroups the 32 columns
    // are contiguous; with four, each warpgroup's 16 sit at the start of its own 32 (then
    // its dS), so K columns 32..63 start 32 TMEM columns in.
    auto gemm_acc = [&](uint32_t d_tmem, uint32_t a_tmem, uint32_t sB, bool accumulate) {
      const uint64_t b0 = make_sdesc_sw128(sB, Plan::kChunkBytes, 1024);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t boff = (uint32_t)(kk * 16 * 128) >> 4;
        const uint32_t aoff = (uint32_t)(8 * kk + (C::kWG == 4 ? 16 * (kk >> 1) : 0));
        ptx::umma_ts_warp(d_tmem, a_tmem + aoff, b0 + boff, idAcc, (accumulate || kk > 0) ? 1u : 0u);
      }
    };
    // Fused form: dQ(step) = dS K over the tile's 128 keys. A is the dS^T tile (rows = keys,
    // queries contiguous: MN-major for M = queries), B the item's K (rows = keys, head dim
    // contiguous: MN-major for N = D); 16 keys (2 KB of rows) per instruction.
    auto gemm_dq = [&](uint32_t d_tmem) {
      const uint64_t a0 = make_sdesc_sw128(sbase + Plan::kDs, Plan::kChunkBytes, 1024);
      const uint64_t b0 = make_sdesc_sw128(sX1, Plan::kChunkBytes, 1024);
#pragma unroll
      for (int kk = 0; kk < kBlockN / 16; ++kk) {
        const uint32_t off = (uint32_t)(kk * 16 * 128) >> 4;
        ptx::umma_ss_warp(d_tmem, a0 + off, b0 + off, idDq, kk > 0 ? 1u : 0u);
      }
    };
    const uint32_t tT1 = tmem + C::kT1;
    const uint32_t tAcc1 = tmem + C::kAcc1, tAcc2 = tmem + C::kAcc2;
    Ring<NS> ring;
    uint32_t x_par = 0, t1f_par = 0, ae_par = 0;
    // Step g uses T2 buffer g % kT2Bufs; its barriers' parity is that of the buffer's use
    // count, g / kT2Bufs.
    auto t2_buf = [](int g) { return C::kT2Bufs == 2 ? (g & 1) : 0; };
    auto t2_use = [](int g) { return (uint32_t)(g / C::kT2Bufs) & 1u; };
    int steps_issued = 0, items_accumulated = 0;
    bool ok = true;
    struct Pending {
      bool valid;
      int st1, st2;
      bool first, last;  // first / last step of its item
      int g;             // the step's index among this CTA's steps
    };
    Pending pend{false, 0, 0, false, false, 0};
    auto acquire = [&]() -> int {
      const int st = ring.stage;
      const uint32_t ph = ring.phase;
      ring.next();
      if (!W.wait_warp(bar(Plan::kRingFull + st), ph)) return -1;
      ptx::tc_fence_after();
      return st;
    };
    // A(step): accumulating GEMMs of a step whose G1, G2 were issued earlier.
    // Fused form: dQ(step) = dS K into the step's dQ buffer. Both halves of dS^T are in
    // shared memory (accumulate() waited for them). At d = 128 accumulate() issues it
    // right after dV and dK (it reuses T2); at d = 64 the main loop issues it after the
    // next step's dP GEMM, which the elementwise warps wait for, and the elementwise warps
    // wait for kDsFree before they overwrite the dS tile.
    auto issue_dq = [&](const Pending& pd) -> bool {
      if constexpr (DQ) {
        const int buf = pd.g % C::kDqBufs;
        if (!C::kDqInT2 && pd.g >= C::kDqBufs) {  // the dQ warps read out this buffer's previous tile
          if (!W.wait_warp(bar(Plan::kDqFree + buf), (uint32_t)(pd.g / C::kDqBufs - 1) & 1u)) return false;
          ptx::tc_fence_after();
        }
        gemm_dq(tmem + (uint32_t)(C::kDq + buf * D));
        ptx::tc_commit_warp(bar(Plan::kDqFull + buf));
        if (!C::kDqInT2) ptx::tc_commit_warp(bar(Plan::kDsFree));
        if (pd.last) ptx::tc_commit_warp(bar(Plan::kXEmpty));  // the dQ GEMM was the last reader of K
      }
      return true;
    };
    auto accumulate = [&](const Pending& pd) -> bool {
      if (pd.first && items_accumulated > 0) {  // the epilogue must have drained the accumulators
        if (!W.wait_warp(bar(Plan::kAccEmpty), ae_par)) return false;
        ae_par ^= 1;
        ptx::tc_fence_after();
      }
      const uint32_t sY1 = sRing + pd.st1 * Plan::kTileBytes;
      const uint32_t sY2 = sRing + pd.st2 * Plan::kTileBytes;
      const int b = t2_buf(pd.g);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        if (!W.wait_warp(bar(Plan::kPdSFull + 2 * b + h), t2_use(pd.g))) return false;
        ptx::tc_fence_after();
        const bool acc = !pd.first || h > 0;
        const uint32_t tP = tmem + (uint32_t)(C::t2_col(b) + 64 * h);
        if (KV) {
          gemm_acc(tAcc2, tP, sY2 + h * kHalfRows, acc);       // dV += P_h^T dO_h
          gemm_acc(tAcc1, tP + C::kCols / 2, sY1 + h * kHalfRows, acc);  // dK += dS_h^T Q_h
        } else {
          gemm_acc(tAcc1, tP, sY1 + h * kHalfRows, acc);       // dQ += dS_h K_h
        }
        ptx::tc_commit_warp(bar(Plan::kT2Free + 2 * b + h));
      }
      // The step's Q and dO tiles are not read after dK and dV.
      ptx::tc_commit_warp(bar(Plan::kRingEmpty + pd.st1));
      if (KV) ptx::tc_commit_warp(bar(Plan::kRingEmpty + pd.st2));
      if (pd.last) {
        ptx::tc_commit_warp(bar(Plan::kAccFull));
        ++items_accumulated;
      }
      if constexpr (C::kDqInT2) {
        // dQ overwrites T2: wait until the dV and dK GEMMs above have read P and dS there.
#pragma unroll 1
        for (int h = 0; h < 2; ++h)
          if (!W.wait_warp(bar(Plan::kT2Free + h), t2_use(pd.g))) return false;
        ptx::tc_fence_after();
        return issue_dq(pd);
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
      // item's epilogue, which waits for the last A(); issue it before waiting for X. Fused
      // form: the last dQ GEMM reads X (K), which is refilled only after it.
      if ((!KV || DQ) && pend.valid) {
        if (!(ok = accumulate(pend))) break;
        if (DQ && !C::kDqInT2 && !(ok = issue_dq(pend))) break;
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
        Pending dq_next{false, 0, 0, false, false, 0};  // d = 64: dQ issued after this dP
        if (pend.valid) {
          if (!(ok = accumulate(pend))) break;
          if (DQ && !C::kDqInT2) dq_next = pend;
          pend.valid = false;
        }
        const int st2 = acquire();
        ok = st2 >= 0;
        if (!ok) break;
        if (kSplitDP) {
          // dP in two column halves: half h of T2 is rewritten as soon as A_h(s-1) finished
          // reading P_h / dS_h from it, and elementwise warpgroup h starts on it at once.
          const int b = t2_buf(steps_issued);
#pragma unroll 1
          for (int h = 0; h < 2 && ok; ++h) {
            if (steps_issued >= C::kT2Bufs) {
              if (C::kDqInT2) {  // the dQ warps read this half of dQ(s-1) out of T2
                if (!(ok = W.wait_warp(bar(Plan::kDqFree + h), (uint32_t)(steps_issued - 1) & 1u))) break;
              } else {  // the accumulating GEMMs of the buffer's previous step are done
                if (!(ok = W.wait_warp(bar(Plan::kT2Free + 2 * b + h), t2_use(steps_issued - C::kT2Bufs)))) break;
              }
              ptx::tc_fence_after();
            }
            gemm_nt(tmem + (uint32_t)(C::t2_col(b) + 64 * h), sX2, tmem + C::kXdO,
                    sRing + st2 * Plan::kTileBytes + h * kHalfRows, idNT64);
            ptx::tc_commit_warp(bar(Plan::kT2Full + 2 * b + h));
          }
          if (!ok) break;
        } else {
          const int b = t2_buf(steps_issued);
          if (steps_issued >= C::kT2Bufs) {
#pragma unroll 1
            for (int h = 0; h < 2 && ok; ++h) {
              if (C::kDqInT2) {
                ok = W.wait_warp(bar(Plan::kDqFree + h), (uint32_t)(steps_issued - 1) & 1u);
              } else {
                ok = W.wait_warp(bar(Plan::kT2Free + 2 * b + h), t2_use(steps_issued - C::kT2Bufs));
              }
            }
            if (!ok) break;
            ptx::tc_fence_after();
          }
          gemm_nt(tmem + (uint32_t)C::t2_col(b), sX2, tmem + C::kXdO, sRing + st2 * Plan::kTileBytes, idNT);
          ptx::tc_commit_warp(bar(Plan::kT2Full + 2 * b));
          ptx::tc_commit_warp(bar(Plan::kT2Full + 2 * b + 1));
        }
        if (dq_next.valid && !(ok = issue_dq(dq_next))) break;
        if (!KV) ptx::tc_commit_warp(bar(Plan::kRingEmpty + st2));  // V: only dP reads it
        if (!DQ && s == it.nsteps - 1) ptx::tc_commit_warp(bar(KV ? Plan::kXEmpty : Plan::kXTFree));  // last reads of X
        pend = Pending{true, st1, st2, s == 0, s == it.nsteps - 1, steps_issued};
        ++steps_issued;
      }
    }
    if (ok && pend.valid) {
      ok = accumulate(pend);
      if (ok && DQ && !C::kDqInT2) ok = issue_dq(pend);
    }
    ptx::tc_commit_warp(bar(Plan::kDrain));
    if (lane == 0) drain_wait(bar(Plan::kDrain), 0, p.timeout_ns, p.status, p.host_flag);
    __syncwarp();
  } else if (DQ && warp >= C::kWarpDq) {
    ptx::setmaxnreg_dec<C::kRegsDq>();
    // ======================================================= dQ reduction ===
    // Per step: the dQ tile of the step's query tile (TMEM, thread = query row) goes out in
    // 32-column chunks through kDqStage shared-memory staging chunks (row r's 128 bytes with
    // the 128-byte swizzle: 16-byte unit u at position u ^ (r & 7), the box layout of tmDq),
    // and each chunk is added into the accumulator by one TMA reduce, issued by one thread.
    // Rows past the map's row extent are dropped by the TMA unit; rows of a packed batch
    // past the sequence's end add exact zeros (their P, hence dS, is 0). The TMEM columns
    // are handed back (DqFree) as soon as they are in registers. Named barrier 1 (these
    // 128 threads) orders the staging writes against the reduce that reads them.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const bool leader = warp == C::kWarpDq && lane == 0;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t stage0 = sbase + Plan::kStage + (uint32_t)r * 128;
    int g = 0;       // steps of this CTA
    int chunks = 0;  // staging chunks filled so far
    bool ok = true;
    ItemReader reader;
    while (ok) {
      int t;
      if (!(ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, true, t)) || t < 0) break;
      const BwdItem it = decode_bwd<KV, WIN, VAR>(t, p);
      if (it.nsteps == 0) continue;  // block past its sequence's end
      const int nq = it.hi - it.lo;
      for (int s = 0; s < it.nsteps && ok; ++s, ++g) {
        const int ytile = it.lo + s % nq;
        const int hy = it.hx * p.kv_group + s / nq;
        const int buf = g % C::kDqBufs;
        if (!(ok = W.wait_warp(bar(Plan::kDqFull + buf), (uint32_t)(g / C::kDqBufs) & 1u))) break;
        ptx::tc_fence_after();
        // Box coordinates in tmDq: (column, row, plane); plane = b * H + h, or h when packed.
        const int y = (VAR ? it.s0 : 0) + ytile * kBlockM;
        const int z = VAR ? hy : it.b * p.H + hy;
        const uint32_t src = tmem + lane_off + (uint32_t)(C::kDq + buf * D);
#pragma unroll 1
        for (int ch = 0; ch < D / 32; ++ch, ++chunks) {
          uint32_t v[32];
          ptx::tmem_ld32(src + ch * 32, v);
          ptx::tmem_wait_ld();
          ptx::reg_fence32(v);
          if (C::kDqInT2 ? (ch & 1) == 1 : ch == D / 32 - 1) {
            ptx::tc_fence_before();  // d = 128: this 64-column half of T2; d = 64: the buffer
            ptx::mbar_arrive(bar(Plan::kDqFree + (C::kDqInT2 ? ch >> 1 : buf)));
          }
          const int sb = chunks % C::kDqStage;
          if (chunks >= C::kDqStage) {  // the reduce that last read chunk sb has read it
            if (leader) ptx::bulk_wait_group_read1();
            ptx::named_bar_sync(1, 128);
          }
          const uint32_t row_addr = stage0 + (uint32_t)sb * Plan::kChunkBytes;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            ptx::st_shared_v4(row_addr + (((uint32_t)u ^ (uint32_t)(r & 7)) << 4), v[4 * u], v[4 * u + 1],
                              v[4 * u + 2], v[4 * u + 3]);
          ptx::fence_proxy_async_smem();
          ptx::named_bar_sync(1, 128);
          if (leader) {
            ptx::tma_reduce_add_3d(&tmDq, sbase + Plan::kStage + (uint32_t)sb * Plan::kChunkBytes, ch * 32, y, z);
            ptx::bulk_commit_group();
          }
        }
      }
    }
    // Every reduce must have read its staging chunk (and landed) before the CTA exits.
    if (leader) ptx::bulk_wait_group0();
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
