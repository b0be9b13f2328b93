// Causal attention forward at d = 128 on CTA pairs: the third forward kernel of this
// library (attn_fwd_pair_kernel), for batched launches without a window.
//
// Same math as mls-bench_fused_attention/fused_attention.py:8-144 (softmax(QK^T * scale) V
// with an optional causal mask, fp32 accumulation, output in the input dtype). It keeps the
// two-sub-tile kernel's per-SM structure (two 128-row query sub-tiles, S and O of both in
// TMEM, P in shared memory, one softmax warpgroup per sub-tile) and runs it on a cluster of
// two CTAs that share every tensor-core instruction:
//
//   * an item is 512 query rows: pair sub-tile i is rows [256 i, 256 i + 256), of which CTA
//     r (cluster rank) holds rows 256 i + 128 r + [0, 128) in its shared memory and TMEM;
//   * rank 0 issues every MMA as a cta_group::2 instruction with M = 256: S_i = Q_i K^T
//     reads each CTA's own Q rows and 64 of the tile's 128 keys from each CTA; O_i += P_i V
//     reads each CTA's own P rows and 64 of V's 128 columns from each CTA. Each CTA
//     therefore loads half of every K and V tile, and the tensor core reads per SM half
//     the B-operand bytes of the one-CTA kernel: ~288 KB of shared-memory traffic per
//     256-row step instead of ~384 KB, and 16 KB ring stages (six instead of three);
//   * completions are committed to both CTAs' barriers (multicast commit); the barriers
//     rank 0's MMA warps wait on (S free, P full, O empty, K/V and Q full) count
//     arrivals and TMA bytes from both CTAs; rank 0 schedules items for both.
//
// Warp roles (512 threads, both CTAs):
//   warps 0-7    softmax: warpgroup i = sub-tile i, thread = query row = TMEM lane
//   warps 8-11   epilogue: O * (1/l) -> bf16/fp16 -> global, fp32 logsumexp
//   warps 12-13  rank 0: MMA issue for sub-tile 0 / 1; warp 12 also allocates TMEM (both)
//   warps 14-15  TMA producers: Q of sub-tile 0 / 1; warp 14 also fills the K/V ring
//                (and, on rank 0, takes items from the work counter and publishes them)
#pragma once

#include "attn_fwd_kernel.cuh"

namespace apex {

struct PairCfg {
  static constexpr int D = 128;
  static constexpr int kNS = 6;          // ring stages: half a K or V tile (16 KB) each
  static constexpr int kThreads = 512;
  static constexpr int kItemRows = 512;  // two pair sub-tiles of 256 rows
  static constexpr int kTmemO = 256;     // S_i at 128 i, O_i at 256 + 128 i
  static constexpr int kRegsSoftmax = 184;
  static constexpr int kRegsEpilogue = 80;
  static constexpr int kRegsOther = 56;
  static_assert(128 * (2 * kRegsSoftmax + kRegsEpilogue + kRegsOther) <= kThreads * (65536 / kThreads),
                "setmaxnreg split exceeds the launch register allocation");
};

struct PairPlan {
  static constexpr int NS = PairCfg::kNS;
  static constexpr int kChunkBytes = kBlockM * 128;     // 128 rows x 64 columns x 2 B, SW128
  static constexpr int kHalfChunkBytes = 64 * 128;      // 64 rows x 64 columns (a K half)
  static constexpr int kQTileBytes = kBlockM * 128 * 2; // one sub-tile of Q (or of P)
  static constexpr int kStageBytes = 16384;             // 64 keys x 128 of K, or 128 keys x 64 of V
  static constexpr int kQ = 0;
  static constexpr int kP = kQ + 2 * kQTileBytes;
  static constexpr int kKV = kP + 2 * kQTileBytes;
  static constexpr int kBars = kKV + NS * kStageBytes;
  static constexpr int kKvFull = 0;
  static constexpr int kKvEmpty = NS;
  static constexpr int kQFull = 2 * NS;
  static constexpr int kQEmpty = kQFull + 2;
  static constexpr int kSFull = kQEmpty + 2;
  static constexpr int kSFree = kSFull + 2;
  static constexpr int kPFull = kSFree + 2;
  static constexpr int kPFree = kPFull + 2;
  static constexpr int kOFull = kPFree + 2;
  static constexpr int kOEmpty = kOFull + 2;
  static constexpr int kLFull = kOEmpty + 2;
  static constexpr int kLEmpty = kLFull + 2;
  static constexpr int kDrain = kLEmpty + 2;
  static constexpr int kItemFull = kDrain + 2;
  static constexpr int kItemEmpty = kItemFull + kItemRing;
  static constexpr int kNumBars = kItemEmpty + kItemRing;
  static constexpr int kRowStats = (kBars + kNumBars * 8 + 15) / 16 * 16;  // float l[2][128], m[2][128]
  static constexpr int kItems = kRowStats + 4 * kBlockM * 4;
  static constexpr int kMisc = kItems + kItemRing * 4;  // tmem base, abort flag
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kMaxDynamic = 232448;
  static constexpr int kDynamicBytes = kBytes + 1024 <= kMaxDynamic ? kBytes + 1024 : kBytes;
  static_assert(kBytes <= kMaxDynamic, "shared-memory plan exceeds 227 KB");
  // Readers of the item ring: rank 0's 8 softmax, 4 epilogue, 2 MMA warps and its second
  // producer; rank 1's 8 softmax, 4 epilogue warps and both producers.
  static constexpr int kItemReaders = 15 + 14;
};

// Bounded waits for barriers that the other CTA of the pair may arrive on (cluster-scope
// acquire); otherwise as Waiter.
struct PairWaiter {
  volatile int* abort_flag;
  int* status;
  unsigned long long timeout_ns;
  int* host_flag;

  __device__ __forceinline__ bool wait(uint32_t bar, uint32_t parity) const {
    if (ptx::mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = ptx::globaltimer_ns();
    while (true) {
#pragma unroll 1
      for (int i = 0; i < 64; ++i)
        if (ptx::mbar_try_wait_cluster(bar, parity)) return true;
      if (*abort_flag) return false;
      if (ptx::globaltimer_ns() - t0 > timeout_ns) {
        *abort_flag = 1;
        report_error(status, host_flag, kStatusWaitTimeout);
        return false;
      }
    }
  }
  __device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity) const {
    return __all_sync(0xffffffffu, wait(bar, parity));
  }
};

struct PairItem {
  int b, h, m0;
  int nb[2];   // K/V tiles of pair sub-tile i (0: no rows)
  int nbmax;
  int nkb, len;
  __device__ __forceinline__ int nbi(int i) const { return i == 0 ? nb[0] : nb[1]; }
};

// Item t -> (b, h, 512-row query block), with the L2 head groups and the longest-first
// order of decode_item.
__device__ __forceinline__ PairItem decode_pair_item(int t, const AttnParams& p) {
  const int MB = p.num_mblocks;
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
  const int mb = MB - 1 - r / size;
  const int bh = base + r % size;
  PairItem it;
  it.b = bh / p.H;
  it.h = bh - it.b * p.H;
  it.m0 = mb * PairCfg::kItemRows;
  it.len = p.N;
  it.nkb = p.num_kblocks;
  for (int i = 0; i < 2; ++i) {
    const int r0 = it.m0 + 256 * i;  // first row of pair sub-tile i (its rank-1 half starts at r0 + 128)
    it.nb[i] = r0 >= p.N ? 0 : (p.causal ? min(it.nkb, (r0 + 128) / kBlockN + 1) : it.nkb);
  }
  it.nbmax = max(it.nb[0], it.nb[1]);
  return it;
}

template <typename T, int EMU8>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairCfg::kThreads, 1)
    attn_fwd_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK64,
                         const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using C = PairCfg;
  using Plan = PairPlan;
  constexpr int D = C::D;
  constexpr int NS = C::kNS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  if (Plan::kDynamicBytes == Plan::kBytes && (raw_addr & 1023u) != 0) {
    // Both CTAs of a pair see the same base, so both return here, before any pair step.
    if (threadIdx.x == 0) report_error(p.status, p.host_flag, kStatusSmemAlign);
    return;
  }
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  const uint32_t sbase = raw_addr + pad;
  uint8_t* smem = smem_raw + pad;

  const uint32_t rank = ptx::cluster_rank();
  const bool leader = rank == 0;
  const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0);
  const int lane = (int)(threadIdx.x & 31);
  constexpr int kWarpEpi = 8;
  constexpr int kWarpMma = 12;
  constexpr int kWarpProd = 14;
  constexpr uint16_t kBoth = 0x3;

  auto bar = [&](int slot) -> uint32_t { return sbase + Plan::kBars + slot * 8; };
  // The same barrier in rank 0's shared memory (shared::cluster window).
  auto lbar = [&](int slot) -> uint32_t { return ptx::mapa(bar(slot), 0); };
  float* row_l = reinterpret_cast<float*>(smem + Plan::kRowStats);  // [2][128]
  float* row_m = row_l + 2 * kBlockM;                                // [2][128]
  int* items = reinterpret_cast<int*>(smem + Plan::kItems);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Plan::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Plan::kMisc + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      ptx::mbar_init(bar(Plan::kKvFull + s), 1);   // rank 0's expect_tx (+ both CTAs' bytes)
      ptx::mbar_init(bar(Plan::kKvEmpty + s), 2);  // one commit per MMA warp
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(bar(Plan::kQFull + i), 1);
      ptx::mbar_init(bar(Plan::kQEmpty + i), 1);
      ptx::mbar_init(bar(Plan::kSFull + i), 1);
      ptx::mbar_init(bar(Plan::kSFree + i), 8);    // 4 softmax warps x 2 CTAs
      ptx::mbar_init(bar(Plan::kPFull + i), 8);
      ptx::mbar_init(bar(Plan::kPFree + i), 1);
      ptx::mbar_init(bar(Plan::kOFull + i), 1);
      ptx::mbar_init(bar(Plan::kOEmpty + i), 8);   // 4 epilogue warps x 2 CTAs
      ptx::mbar_init(bar(Plan::kLFull + i), kBlockM);
      ptx::mbar_init(bar(Plan::kLEmpty + i), kBlockM);
      ptx::mbar_init(bar(Plan::kDrain + i), 1);
    }
    for (int k = 0; k < kItemRing; ++k) {
      ptx::mbar_init(bar(Plan::kItemFull + k), 1);
      ptx::mbar_init(bar(Plan::kItemEmpty + k), Plan::kItemReaders);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kWarpMma) {
    ptx::tmem_alloc_pair(ptx::smem_u32(tmem_holder), 512);
    ptx::tmem_relinquish_pair();
  }
  if (warp == kWarpProd && lane == 0) {
    ptx::prefetch_tmap(&tmQ);
    ptx::prefetch_tmap(&tmK64);
    ptx::prefetch_tmap(&tmV);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();  // both CTAs' barriers are initialised before either uses the other's
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const PairWaiter W{abort_flag, p.status, p.timeout_ns, p.host_flag};

  // Reader side of the item ring: wait for this CTA's slot, release rank 0's.
  int reads = 0;
  auto read_item = [&](bool whole_warp, int& t) -> bool {
    const int slot = reads % kItemRing;
    const uint32_t parity = (uint32_t)(reads / kItemRing) & 1u;
    ++reads;
    if (whole_warp) {
      if (!W.wait_warp(bar(Plan::kItemFull + slot), parity)) return false;
      t = items[slot];
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_remote(lbar(Plan::kItemEmpty + slot));
    } else {
      if (!W.wait(bar(Plan::kItemFull + slot), parity)) return false;
      t = items[slot];
      ptx::mbar_arrive_remote(lbar(Plan::kItemEmpty + slot));
    }
    return true;
  };

  if (warp < kWarpEpi) {
    // =========================================================== softmax ===
    ptx::setmaxnreg_inc<C::kRegsSoftmax>();
    const int i = warp >> 2;            // sub-tile
    const int quarter = warp & 3;       // TMEM lane quarter
    const int r = quarter * 32 + lane;  // row within the sub-tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off + (uint32_t)(i * 128);
    const uint32_t tO = tmem + lane_off + (uint32_t)(C::kTmemO + i * D);
    // Row r of P: two 16 KB chunks (keys 0-63, 64-127) of the SW128 K-major layout; 16-byte
    // unit u of the row sits at unit position u ^ (r & 7).
    const uint32_t sP = sbase + Plan::kP + i * Plan::kQTileBytes + r * 128;
    const float c = p.scale_log2;
    const float2 c2 = make_float2(c, c);
    uint32_t s_par = 0, le_par = 1, pf_par = 0;
    int p_written = 0;
    bool ok = true;
    while (ok) {
      int t;
      if (!(ok = read_item(true, t)) || t < 0) break;
      const PairItem it = decode_pair_item(t, p);
      const int nb = it.nbi(i);
      if (nb == 0) continue;
      const int r0 = it.m0 + 256 * i + 128 * (int)rank;  // first row of this CTA's sub-tile
      const int diag = r0 / kBlockN;
      float m = 0.f, l = 0.f;
      for (int j = 0; j < nb; ++j) {
        if (!(ok = W.wait_warp(bar(Plan::kSFull + i), s_par))) break;
        s_par ^= 1;
        ptx::tc_fence_after();
        float s[kBlockN];
        {
          uint32_t v[4][32];
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) ptx::tmem_ld32(tS + ch * 32, v[ch]);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            ptx::reg_fence32(v[ch]);
#pragma unroll
            for (int e = 0; e < 32; ++e) s[ch * 32 + e] = __uint_as_float(v[ch][e]);
          }
        }
        // S is in registers: rank 0 may compute the next S into this buffer.
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive_remote(lbar(Plan::kSFree + i));
        // Causal: the diagonal tile masks keys past the row; rank 0's rows see no key of
        // the pair sub-tile's last tile (rank 1's diagonal), which is then masked whole.
        const bool diag_tile = p.causal && j >= diag;
        const int kv_last_valid = it.len - (it.nkb - 1) * kBlockN;
        const bool tail_tile = !p.causal && j == it.nkb - 1 && kv_last_valid < kBlockN;
        const bool masked = diag_tile || tail_tile;  // warp-uniform
        if (masked) {
          const int kv_limit = diag_tile ? (j == diag ? r + 1 : 0) : kv_last_valid;
#pragma unroll
          for (int e = 0; e < kBlockN; ++e)
            if (e >= kv_limit) s[e] = -INFINITY;
        }
        float mx0 = fmaxf(s[0], s[1]), mx1 = fmaxf(s[2], s[3]);
        float mx2 = fmaxf(s[4], s[5]), mx3 = fmaxf(s[6], s[7]);
#pragma unroll
        for (int e = 8; e < kBlockN; e += 8) {
          mx0 = ptx::fmax3(mx0, s[e], s[e + 1]);
          mx1 = ptx::fmax3(mx1, s[e + 2], s[e + 3]);
          mx2 = ptx::fmax3(mx2, s[e + 4], s[e + 5]);
          mx3 = ptx::fmax3(mx3, s[e + 6], s[e + 7]);
        }
        const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * c;  // log2 domain
        float alpha = 1.f;
        bool resc = false;
        if (j == 0) {
          m = mx;  // tile 0 always holds key 0, which every row sees
        } else if (mx > m + kRescaleLog2) {
          alpha = ptx::ex2(m - mx);
          m = mx;
          resc = true;
        }
        l *= alpha;
        const float2 nm2 = make_float2(-m, -m);
        float2 sa = make_float2(0.f, 0.f), sb = make_float2(0.f, 0.f);
        uint32_t pk[2][32];
        auto exp_half = [&](const int half, auto poly) {
          constexpr bool kPoly = decltype(poly)::value;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float2 x = __ffma2_rn(make_float2(s[half * 64 + 2 * e], s[half * 64 + 2 * e + 1]), c2, nm2);
            float2 pr;
            if (kPoly && (e & 7) < EMU8) pr = exp2_poly_pair(x);
            else pr = make_float2(ptx::ex2(x.x), ptx::ex2(x.y));
            if (e & 1) sb = __fadd2_rn(sb, pr);
            else sa = __fadd2_rn(sa, pr);
            pk[half][e] = DType<T>::pack(pr.x, pr.y);
          }
        };
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (masked) exp_half(h, std::false_type{});  // masked keys hold -inf: MUFU gives exactly 0
          else exp_half(h, std::integral_constant<bool, (EMU8 > 0)>{});
        }
        const float2 sum = __fadd2_rn(sa, sb);
        l += sum.x + sum.y;
        // The P buffer and O are free once the previous P.V of this sub-tile completed.
        if (p_written > 0) {
          if (!(ok = W.wait_warp(bar(Plan::kPFree + i), pf_par))) break;
          pf_par ^= 1;
        }
        ++p_written;
        ptx::tc_fence_after();
        if (__any_sync(0xffffffffu, resc)) {
          // O is quiescent: the previous P.V completed (above) and the next waits for P.
#pragma unroll 1
          for (int ch = 0; ch < D / 32; ++ch) {
            uint32_t v[32];
            ptx::tmem_ld32(tO + ch * 32, v);
            ptx::tmem_wait_ld();
            ptx::reg_fence32(v);
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
            ptx::tmem_st32(tO + ch * 32, v);
          }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int u = 0; u < 8; ++u)
            ptx::st_shared_v4(sP + h * Plan::kChunkBytes + ((u ^ (r & 7)) << 4), pk[h][4 * u], pk[h][4 * u + 1],
                              pk[h][4 * u + 2], pk[h][4 * u + 3]);
        ptx::fence_proxy_async_smem();
        ptx::tmem_wait_st();  // the O rescale stores, if any
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive_remote(lbar(Plan::kPFull + i));
      }
      if (!ok) break;
      if (!(ok = W.wait_warp(bar(Plan::kLEmpty + i), le_par))) break;
      le_par ^= 1;
      row_l[i * kBlockM + r] = l;
      row_m[i * kBlockM + r] = m;
      ptx::mbar_arrive(bar(Plan::kLFull + i));
    }
  } else if (warp < kWarpMma) {
    // ========================================================== epilogue ===
    ptx::setmaxnreg_dec<C::kRegsEpilogue>();
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint32_t lf_par = 0, of_par = 0;  // bit i: barrier parity for sub-tile i
    auto finish = [&](const PairItem& it, const int i) -> bool {
      if (!W.wait_warp(bar(Plan::kLFull + i), (lf_par >> i) & 1u)) return false;
      lf_par ^= 1u << i;
      const float l = row_l[i * kBlockM + r];
      const float m = row_m[i * kBlockM + r];
      ptx::mbar_arrive(bar(Plan::kLEmpty + i));
      if (!W.wait_warp(bar(Plan::kOFull + i), (of_par >> i) & 1u)) return false;
      of_par ^= 1u << i;
      ptx::tc_fence_after();
      const float inv = 1.f / l;
      const int row = it.m0 + 256 * i + 128 * (int)rank + r;
      const bool valid = row < it.len;
      T* orow = reinterpret_cast<T*>(p.o) + (long long)it.b * p.o_sb + (long long)it.h * p.o_sh +
                (long long)row * p.o_sn;
      const uint32_t tO = tmem + lane_off + (uint32_t)(C::kTmemO + i * D);
#pragma unroll 1
      for (int ch = 0; ch < D / 32; ++ch) {
        uint32_t v[32];
        ptx::tmem_ld32(tO + ch * 32, v);
        ptx::tmem_wait_ld();
        ptx::reg_fence32(v);
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          pk[e] = DType<T>::pack(__uint_as_float(v[2 * e]) * inv, __uint_as_float(v[2 * e + 1]) * inv);
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + ch * 32);
#pragma unroll
          for (int w = 0; w < 4; ++w) dst[w] = make_uint4(pk[4 * w], pk[4 * w + 1], pk[4 * w + 2], pk[4 * w + 3]);
        }
      }
      // O is in registers: rank 0 may start the next item's P.V into it.
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_remote(lbar(Plan::kOEmpty + i));
      if (p.lse != nullptr && valid)
        p.lse[((long long)it.b * p.H + it.h) * p.N + row] = (m + __log2f(l)) * 0.69314718055994531f;
      return true;
    };
    bool ok = true;
    while (ok) {
      int t;
      if (!(ok = read_item(true, t)) || t < 0) break;
      const PairItem it = decode_pair_item(t, p);
      for (int i = 0; i < 2 && ok; ++i)
        if (it.nbi(i) > 0) ok = finish(it, i);
    }
  } else {
    ptx::setmaxnreg_dec<C::kRegsOther>();
    if (warp < kWarpProd) {
      if (leader) {
        // =============================================================== MMA ===
        // Warp i issues every pair MMA of sub-tile i: S_i(j) once both CTAs' softmax read
        // S_i(j - 1), O_i += P_i(j) V(j) once both wrote P_i(j). Both warps walk every ring
        // stage (the stage sequence of the two-sub-tile kernel: K(0); K(j + 1), V(j)).
        const int i = warp - kWarpMma;
        constexpr uint32_t idS = make_idesc<T>(256, kBlockN, false);
        constexpr uint32_t idPV = make_idesc<T>(256, D, true);
        const uint32_t sQ = sbase + Plan::kQ + i * Plan::kQTileBytes;
        const uint32_t sKV = sbase + Plan::kKV;
        const uint32_t sPi = sbase + Plan::kP + i * Plan::kQTileBytes;
        const uint32_t tSi = tmem + (uint32_t)(i * 128);
        const uint32_t tOi = tmem + (uint32_t)(C::kTmemO + i * D);
        Ring<NS> ring;
        uint32_t q_par = 0, sf_par = 0, pf_par = 0, oe_par = 0;
        int s_issued = 0;
        bool first_item = true;
        bool ok = true;
        auto acquire = [&]() -> int {
          const int st = ring.stage;
          const uint32_t ph = ring.phase;
          ring.next();
          if (!W.wait_warp(bar(Plan::kKvFull + st), ph)) return -1;
          ptx::tc_fence_after();
          return st;
        };
        auto do_S = [&](bool needed) -> bool {
          if (needed && s_issued > 0) {
            if (!W.wait_warp(bar(Plan::kSFree + i), sf_par)) return false;
            sf_par ^= 1;
          }
          const int st = acquire();
          if (st < 0) return false;
          if (needed) {
            const uint64_t a0 = make_sdesc_sw128(sQ, 16, 1024);
            const uint64_t b0 = make_sdesc_sw128(sKV + st * Plan::kStageBytes, 16, 1024);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t aoff = (uint32_t)((kk >> 2) * Plan::kChunkBytes + (kk & 3) * 32) >> 4;
              const uint32_t boff = (uint32_t)((kk >> 2) * Plan::kHalfChunkBytes + (kk & 3) * 32) >> 4;
              ptx::umma_ss_pair_warp(tSi, a0 + aoff, b0 + boff, idS, kk > 0 ? 1u : 0u);
            }
          }
          ptx::tc_commit_pair_warp(bar(Plan::kKvEmpty + st), kBoth);
          if (needed) {
            ptx::tc_commit_pair_warp(bar(Plan::kSFull + i), kBoth);
            ++s_issued;
          }
          return true;
        };
        auto do_PV = [&](bool needed, bool first, bool last) -> bool {
          if (needed) {
            if (first && !first_item) {  // both epilogues must have drained O_i
              if (!W.wait_warp(bar(Plan::kOEmpty + i), oe_par)) return false;
              oe_par ^= 1;
            }
            if (!W.wait_warp(bar(Plan::kPFull + i), pf_par)) return false;
            pf_par ^= 1;
          }
          const int st = acquire();
          if (st < 0) return false;
          if (needed) {
            const uint64_t b0 = make_sdesc_sw128(sKV + st * Plan::kStageBytes, Plan::kChunkBytes, 1024);
#pragma unroll
            for (int kk = 0; kk < kBlockN / 16; ++kk) {
              const uint32_t boff = (uint32_t)(kk * 16 * 128) >> 4;
              const uint64_t a = make_sdesc_sw128(sPi + (kk >> 2) * Plan::kChunkBytes + (kk & 3) * 32, 16, 1024);
              ptx::umma_ss_pair_warp(tOi, a, b0 + boff, idPV, (!first || kk > 0) ? 1u : 0u);
            }
          }
          ptx::tc_commit_pair_warp(bar(Plan::kKvEmpty + st), kBoth);
          if (needed) {
            ptx::tc_commit_pair_warp(bar(Plan::kPFree + i), kBoth);
            if (last) ptx::tc_commit_pair_warp(bar(Plan::kOFull + i), kBoth);
          }
          return true;
        };
        while (ok) {
          int t;
          if (!(ok = read_item(true, t)) || t < 0) break;
          const PairItem it = decode_pair_item(t, p);
          const int nb = it.nbi(i);
          if (nb > 0) {
            if (!(ok = W.wait_warp(bar(Plan::kQFull + i), q_par))) break;
            q_par ^= 1;
          }
          if (it.nbmax > 0) ok = do_S(nb > 0);
          if (ok && nb == 1) ptx::tc_commit_pair_warp(bar(Plan::kQEmpty + i), kBoth);  // last use of Q_i
          for (int j = 0; j < it.nbmax && ok; ++j) {
            if (j + 1 < it.nbmax) {
              ok = do_S(j + 1 < nb);
              if (ok && nb > 0 && j + 2 == nb) ptx::tc_commit_pair_warp(bar(Plan::kQEmpty + i), kBoth);
            }
            if (ok) ok = do_PV(j < nb, j == 0, j == nb - 1);
          }
          if (nb > 0) first_item = false;
        }
        // Every pair MMA (and its commit arrivals, in both CTAs) lands before either CTA
        // releases TMEM or shared memory: rank 1 passes the final cluster barrier only
        // after this wait.
        ptx::tc_commit_pair_warp(bar(Plan::kDrain + i), kBoth);
        if (lane == 0) drain_wait(bar(Plan::kDrain + i), 0, p.timeout_ns, p.status, p.host_flag);
        __syncwarp();
      }
    } else {
      // ========================================================= producers ===
      // Producer q loads this CTA's rows of Q sub-tile q; producer 0 also loads this CTA's
      // half of every K/V stage. All completions count on rank 0's barriers, whose
      // expect_tx (rank 0's producers) covers both CTAs' bytes. Rank 0's producer 0 takes
      // items from the work counter and publishes them to both CTAs' item rings.
      if (lane == 0) {
        const int qi = warp - kWarpProd;
        const uint64_t pol_q = ptx::policy_evict_first();
        const uint64_t pol_kv = ptx::policy_evict_last();
        const uint32_t sQ = sbase + Plan::kQ + qi * Plan::kQTileBytes;
        const uint32_t sKV = sbase + Plan::kKV;
        const bool scheduler = leader && qi == 0;
        Ring<NS> ring;
        uint32_t qe_par = 1;
        int fills = 0, q_fills = 0;
        bool ok = true;
        auto fill = [&](bool is_k, int j, int hkv, int b) -> bool {
          const int st = ring.stage;
          const uint32_t ph = ring.phase;
          ring.next();
          if (!W.wait(bar(Plan::kKvEmpty + st), ph ^ 1)) return false;
          if (leader) ptx::mbar_arrive_expect_tx(bar(Plan::kKvFull + st), (uint32_t)(2 * Plan::kStageBytes));
          const uint32_t dst = sKV + st * Plan::kStageBytes;
          if (is_k) {  // keys [128 j + 64 rank, +64), all 128 columns
            for (int cc = 0; cc < 2; ++cc)
              ptx::tma_load_4d_pair(dst + cc * Plan::kHalfChunkBytes, &tmK64, lbar(Plan::kKvFull + st), cc * 64,
                                    j * kBlockN + 64 * (int)rank, hkv, b, pol_kv);
          } else {  // all 128 keys of tile j, columns [64 rank, +64)
            ptx::tma_load_4d_pair(dst, &tmV, lbar(Plan::kKvFull + st), 64 * (int)rank, j * kBlockN, hkv, b, pol_kv);
          }
          ++fills;
          return true;
        };
        int fetched = scheduler ? atomicAdd(p.work_counter, 1) : 0;
        int published = 0;
        while (ok) {
          int t;
          if (scheduler) {
            const int slot = published % kItemRing;
            const uint32_t parity = ((uint32_t)(published / kItemRing) & 1u) ^ 1u;
            if (!(ok = W.wait(bar(Plan::kItemEmpty + slot), parity))) break;
            t = fetched < p.num_items ? fetched : -1;
            if (t >= 0) fetched = atomicAdd(p.work_counter, 1);
            items[slot] = t;
            ptx::st_cluster_u32(ptx::mapa(ptx::smem_u32(items + slot), 1), (uint32_t)t);
            ptx::mbar_arrive_cluster(ptx::mapa(bar(Plan::kItemFull + slot), 0));
            ptx::mbar_arrive_cluster(ptx::mapa(bar(Plan::kItemFull + slot), 1));
            ++published;
          } else if (!(ok = read_item(false, t))) {
            break;
          }
          if (t < 0) break;
          const PairItem it = decode_pair_item(t, p);
          if (it.nbi(qi) > 0) {
            if (!(ok = W.wait(bar(Plan::kQEmpty + qi), qe_par))) break;
            qe_par ^= 1;
            if (leader) ptx::mbar_arrive_expect_tx(bar(Plan::kQFull + qi), (uint32_t)(2 * Plan::kQTileBytes));
            for (int cc = 0; cc < D / 64; ++cc)
              ptx::tma_load_4d_pair(sQ + cc * Plan::kChunkBytes, &tmQ, lbar(Plan::kQFull + qi), cc * 64,
                                    it.m0 + 256 * qi + 128 * (int)rank, it.h, it.b, pol_q);
            ++q_fills;
          }
          if (qi != 0) continue;
          const int hkv = it.h / p.kv_group;
          if (it.nbmax > 0) ok = fill(true, 0, hkv, it.b);
          for (int j = 0; j < it.nbmax && ok; ++j) {
            if (j + 1 < it.nbmax) ok = fill(true, j + 1, hkv, it.b);
            if (ok) ok = fill(false, j, hkv, it.b);
          }
        }
        // Rank 0's full barriers complete only when both CTAs' loads landed: let every load
        // of the pair land before either CTA exits (rank 1 waits at the cluster barrier).
        if (leader) {
          const int last = fills < NS ? fills : NS;
          for (int k = 0; k < last; ++k) {
            const int f = fills - 1 - k;
            drain_wait(bar(Plan::kKvFull + (f % NS)), (uint32_t)((f / NS) & 1), p.timeout_ns, p.status, p.host_flag);
          }
          if (q_fills > 0) drain_wait(bar(Plan::kQFull + qi), qe_par, p.timeout_ns, p.status, p.host_flag);
        }
      }
      __syncwarp();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();  // neither CTA leaves while the other may still touch its memory
  if (warp == kWarpMma) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem, 512);
  }
}

}  // namespace apex
