// Causal attention forward for sm_100a with one 128-row query tile per CTA and every
// intermediate in TMEM: the second forward kernel of this library, used for head dims 64
// and 128 (batched, optionally grouped-query) in place of attn_fwd_sm100_kernel.
//
// Same math as mls-bench_fused_attention/fused_attention.py:8-144 (softmax(QK^T * scale) V
// with an optional causal mask, fp32 accumulation, output in the input dtype), with a
// buffer plan chosen for the B200's shared-memory bandwidth:
//
//   * TMEM holds two S buffers, two P buffers and O (512 columns at d = 128). S(t+1) is
//     computed while the softmax works on S(t), and P(t) is written while P(t-1) V(t-1)
//     runs, so neither the softmax nor the tensor core waits for the other's round trip.
//   * P V reads P from TMEM (tcgen05.mma with A in tensor memory), so per 128-key tile
//     the tensor core reads only K and V from shared memory. The two-sub-tile kernel
//     keeps P in shared memory at d = 128 and reads it there, which makes shared memory
//     its limit: per tile it moved ~1.5x the bytes this kernel moves.
//   * Two softmax warpgroups split the tile's rows: in each 32-lane TMEM quarter, the
//     warp of warpgroup 0 takes lanes 0-15 and the warp of warpgroup 1 lanes 16-31
//     (16-lane tcgen05.ld/st shapes; four threads share a row and reduce its max with two
//     shuffles). The warpgroups never wait for each other, so one's exponentials overlap
//     the other's loads, row maxima and P stores. A split by key columns would need a
//     row-max exchange every tile, which keeps the two in lockstep: measured, that left
//     the exponential unit idle through every non-exponential phase (45 % busy at d = 64).
//   * A separate epilogue warpgroup normalises O and writes it with TMA tensor stores,
//     staging through the shared-memory Q buffer its item no longer needs.
//   * The MMA warp walks one continuous stream of (item, K/V tile) steps: S of the next
//     item's first tile is issued before P V of the current item's last tile, so item
//     changes cost the softmax no bubble. The producer loads the next item's Q into the
//     second Q buffer ahead of time.
//
// Warp roles (512 threads):
//   warps 0-7    softmax: warp w handles rows 32(w % 4) + 16(w / 4) + [0, 16) of the tile,
//                all 128 keys; thread t holds rows +t/4 and +t/4+8, 32 keys of each
//   warps 8-11   epilogue: O * (1/l) -> bf16/fp16 -> shared memory -> TMA store; fp32 lse
//   warp 12      tcgen05.mma issue (one elected lane) and TMEM allocation
//   warp 13      scheduler and TMA producer (lane 0)
//   warps 14-15  no work; they complete the fourth warpgroup for setmaxnreg
#pragma once

#include "attn_fwd_kernel.cuh"

namespace apex {

template <int D>
struct TileCfg {
  static_assert(D == 64 || D == 128, "the tile kernel covers head dims 64 and 128");
  static constexpr int kNS = D == 64 ? 8 : 4;  // K/V ring stages (one 128-key K or V tile each)
  static constexpr int kThreads = 512;
  // TMEM columns: S_b at 128 b (b = 0, 1), P_b at 256 + 64 b, O at 384.
  static constexpr int kTmemS = 0;
  static constexpr int kTmemP = 256;
  static constexpr int kTmemO = 384;
  static_assert(kTmemO + D <= 512, "TMEM plan overflows 512 columns");
  // setmaxnreg budgets: two softmax warpgroups, the epilogue, the MMA/producer warpgroup.
  static constexpr int kRegsSoftmax = 184;
  static constexpr int kRegsEpilogue = 88;
  static constexpr int kRegsOther = 56;
  static_assert(128 * (2 * kRegsSoftmax + kRegsEpilogue + kRegsOther) <= kThreads * (65536 / kThreads),
                "setmaxnreg split exceeds the launch register allocation");
};

template <int D>
struct TilePlan {
  using C = TileCfg<D>;
  static constexpr int NS = C::kNS;
  static constexpr int kChunkBytes = kBlockM * 128;   // 128 rows x 64 columns x 2 bytes, SW128
  static constexpr int kQBytes = kBlockM * D * 2;     // one Q tile (also one O staging tile)
  static constexpr int kStageBytes = kBlockN * D * 2; // one K or V tile
  static constexpr int kQ = 0;                        // two Q buffers
  static constexpr int kKV = kQ + 2 * kQBytes;
  static constexpr int kBars = kKV + NS * kStageBytes;
  // barrier slots
  static constexpr int kKvFull = 0;
  static constexpr int kKvEmpty = NS;
  static constexpr int kQFull = 2 * NS;         // [2]
  static constexpr int kQEmpty = kQFull + 2;    // [2]
  static constexpr int kSFull = kQEmpty + 2;    // [2]
  static constexpr int kSFree = kSFull + 2;     // [2]
  static constexpr int kPFull = kSFree + 2;     // [2]
  static constexpr int kPFree = kPFull + 2;     // [2]
  static constexpr int kOFull = kPFree + 2;
  static constexpr int kOEmpty = kOFull + 1;
  static constexpr int kLFull = kOEmpty + 1;
  static constexpr int kLEmpty = kLFull + 1;
  static constexpr int kStaged = kLEmpty + 1;   // epilogue: O tile written to the staging buffer
  static constexpr int kDrain = kStaged + 1;
  static constexpr int kItemFull = kDrain + 1;  // [kItemRing]
  static constexpr int kItemEmpty = kItemFull + kItemRing;
  static constexpr int kNumBars = kItemEmpty + kItemRing;
  // float l[128] (row sums), m[128] (row maxima, log2 units): softmax -> epilogue
  static constexpr int kRowStats = (kBars + kNumBars * 8 + 15) / 16 * 16;
  static constexpr int kItems = kRowStats + 2 * kBlockM * 4;
  static constexpr int kMisc = kItems + kItemRing * 4;  // tmem base, abort flag
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kMaxDynamic = 232448;
  static constexpr int kDynamicBytes = kBytes + 1024 <= kMaxDynamic ? kBytes + 1024 : kBytes;
  static_assert(kBytes <= kMaxDynamic, "shared-memory plan exceeds 227 KB");
};

// EMU8: of every 8 exponential pairs of an unmasked tile, how many use the FMA-pipe
// polynomial instead of MUFU.
template <int D, typename T, int EMU8>
__global__ void __launch_bounds__(TileCfg<D>::kThreads, 1)
    attn_fwd_tile_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                         const AttnParams p) {
  using C = TileCfg<D>;
  using Plan = TilePlan<D>;
  constexpr int NS = C::kNS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  if (Plan::kDynamicBytes == Plan::kBytes && (raw_addr & 1023u) != 0) {
    if (threadIdx.x == 0) report_error(p.status, p.host_flag, kStatusSmemAlign);
    return;
  }
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  const uint32_t sbase = raw_addr + pad;
  uint8_t* smem = smem_raw + pad;

  const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0);
  const int lane = (int)(threadIdx.x & 31);
  constexpr int kWarpEpi = 8;
  constexpr int kWarpMma = 12;
  constexpr int kWarpProd = 13;

  auto bar = [&](int slot) -> uint32_t { return sbase + Plan::kBars + slot * 8; };
  float* row_l = reinterpret_cast<float*>(smem + Plan::kRowStats);  // [128]
  float* row_m = row_l + kBlockM;                                    // [128]
  int* items = reinterpret_cast<int*>(smem + Plan::kItems);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Plan::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Plan::kMisc + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      ptx::mbar_init(bar(Plan::kKvFull + s), 1);
      ptx::mbar_init(bar(Plan::kKvEmpty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar(Plan::kQFull + b), 1);
      ptx::mbar_init(bar(Plan::kQEmpty + b), 2);  // last S of the item (commit) + epilogue staging done
      ptx::mbar_init(bar(Plan::kSFull + b), 1);
      ptx::mbar_init(bar(Plan::kSFree + b), 8);   // one arrival per softmax warp
      ptx::mbar_init(bar(Plan::kPFull + b), 8);
      ptx::mbar_init(bar(Plan::kPFree + b), 1);
    }
    ptx::mbar_init(bar(Plan::kOFull), 1);
    ptx::mbar_init(bar(Plan::kOEmpty), 4);        // one arrival per epilogue warp
    ptx::mbar_init(bar(Plan::kLFull), 2 * kBlockM);
    ptx::mbar_init(bar(Plan::kLEmpty), kBlockM);
    ptx::mbar_init(bar(Plan::kStaged), 4);
    ptx::mbar_init(bar(Plan::kDrain), 1);
    // Readers of the item ring: 8 softmax warps, 4 epilogue warps, the MMA warp.
    for (int k = 0; k < kItemRing; ++k) {
      ptx::mbar_init(bar(Plan::kItemFull + k), 1);
      ptx::mbar_init(bar(Plan::kItemEmpty + k), 13);
    }
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kWarpMma) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), 512);
    ptx::tmem_relinquish();
  }
  if (warp == kWarpProd && lane == 0) {
    ptx::prefetch_tmap(&tmQ);
    ptx::prefetch_tmap(&tmK);
    ptx::prefetch_tmap(&tmV);
    ptx::prefetch_tmap(&tmO);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const Waiter W{abort_flag, p.status, p.timeout_ns, p.host_flag};

  if (warp < kWarpEpi) {
    // =========================================================== softmax ===
    ptx::setmaxnreg_inc<C::kRegsSoftmax>();
    const int lb = (warp & 3) * 32 + (warp >> 2) * 16;  // first TMEM lane (= tile row) of this warp
    const int ra = lb + (lane >> 2);                    // this thread's rows: ra and ra + 8
    const int kq = 2 * (lane & 3);                      // its keys: 8e + kq + {0, 1}, e = 0..15
    const uint32_t lane_off = (uint32_t)lb << 16;
    const float sc = p.scale_log2;
    const float2 c2 = make_float2(sc, sc);
    uint32_t le_par = 1;
    int t = 0;  // tiles processed by this CTA (S and P buffer = t & 1)
    bool ok = true;
    ItemReader reader;
    while (ok) {
      int item;
      if (!(ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, true, item)) || item < 0) break;
      const WorkItem it = decode_item<1, false, false>(item, p);
      const int nb = it.nb[0];
      const int diag = it.m0 / kBlockN;
      float m[2] = {0.f, 0.f}, l[2] = {0.f, 0.f};  // rows ra, ra + 8 (log2-domain max, partial sum)
      for (int j = 0; j < nb; ++j, ++t) {
        const int sb = t & 1;
        if (!(ok = W.wait_warp(bar(Plan::kSFull + sb), (uint32_t)(t >> 1) & 1u))) break;
        ptx::tc_fence_after();
        // s[row][2e + b] = S(row, key 8e + kq + b)
        float s[2][32];
        {
          uint32_t v[2][32];
          const uint32_t tS = tmem + lane_off + (uint32_t)(C::kTmemS + sb * 128);
          ptx::tmem_ld_16x256b_x8(tS, v[0]);
          ptx::tmem_ld_16x256b_x8(tS + 64, v[1]);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            ptx::reg_fence32(v[h]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              s[0][16 * h + 2 * i] = __uint_as_float(v[h][4 * i]);
              s[0][16 * h + 2 * i + 1] = __uint_as_float(v[h][4 * i + 1]);
              s[1][16 * h + 2 * i] = __uint_as_float(v[h][4 * i + 2]);
              s[1][16 * h + 2 * i + 1] = __uint_as_float(v[h][4 * i + 3]);
            }
          }
        }
        // S is in registers: the MMA warp may compute S(t + 2) into this buffer.
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(Plan::kSFree + sb));
        const bool diag_tile = p.causal && j == diag;
        const int kv_last_valid = it.len - (it.nkb - 1) * kBlockN;
        const bool tail_tile = !p.causal && j == it.nkb - 1 && kv_last_valid < kBlockN;
        if (diag_tile || tail_tile) {  // warp-uniform
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            const int limit = diag_tile ? ra + 8 * rr + 1 : kv_last_valid;  // keys >= limit are masked
#pragma unroll
            for (int e = 0; e < 16; ++e)
#pragma unroll
              for (int b = 0; b < 2; ++b)
                if (8 * e + kq + b >= limit) s[rr][2 * e + b] = -INFINITY;
          }
        }
        bool resc = false;
        float alpha[2] = {1.f, 1.f};
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          float m0 = fmaxf(s[rr][0], s[rr][1]), m1 = fmaxf(s[rr][2], s[rr][3]);
#pragma unroll
          for (int e = 4; e < 32; e += 4) {
            m0 = ptx::fmax3(m0, s[rr][e], s[rr][e + 1]);
            m1 = ptx::fmax3(m1, s[rr][e + 2], s[rr][e + 3]);
          }
          float mx = fmaxf(m0, m1);
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));  // the four threads of the row
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          mx *= sc;  // log2 domain
          if (j == 0) {
            m[rr] = mx;
          } else if (mx > m[rr] + kRescaleLog2) {
            alpha[rr] = ptx::ex2(m[rr] - mx);
            m[rr] = mx;
            resc = true;
          }
          l[rr] *= alpha[rr];
        }
        // p = exp2(s * c - m), packed to 16-bit pairs in the 16x128b store layout:
        // pk[2e + rr] = P(row ra + 8 rr, keys 8e + kq, 8e + kq + 1)
        uint32_t pk[32];
        float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        auto exps = [&](auto poly) {
          constexpr bool kPoly = decltype(poly)::value;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
              const float2 x = __ffma2_rn(make_float2(s[rr][2 * e], s[rr][2 * e + 1]), c2,
                                          make_float2(-m[rr], -m[rr]));
              float2 pr;
              if (kPoly && ((2 * e + rr) & 7) < EMU8) pr = exp2_poly_pair(x);
              else pr = make_float2(ptx::ex2(x.x), ptx::ex2(x.y));
              acc[rr] = __fadd2_rn(acc[rr], pr);
              pk[2 * e + rr] = DType<T>::pack(pr.x, pr.y);
            }
          }
        };
        if (diag_tile || tail_tile) exps(std::false_type{});  // masked keys hold -inf: MUFU gives exactly 0
        else exps(std::integral_constant<bool, (EMU8 > 0)>{});
        l[0] += acc[0].x + acc[0].y;
        l[1] += acc[1].x + acc[1].y;
        const int pb = t & 1;
        // P buffer pb is free: P(t - 2) V(t - 2) was issued before S(t) by the same thread,
        // so the commit that completed S(t) covered it.
        if (__any_sync(0xffffffffu, resc)) {
          // Rescale these rows of O. O must be quiescent: P(t - 1) V(t - 1), the last MMA
          // into O so far, completed (P(t) V(t) waits for the P written below). j > 0, so
          // tile t - 1 belongs to this item.
          if (!(ok = W.wait_warp(bar(Plan::kPFree + (pb ^ 1)), (uint32_t)((t - 1) >> 1) & 1u))) break;
          ptx::tc_fence_after();
          const uint32_t tO = tmem + lane_off + (uint32_t)C::kTmemO;
#pragma unroll 1
          for (int ch = 0; ch < D / 64; ++ch) {
            uint32_t v[32];
            ptx::tmem_ld_16x256b_x8(tO + ch * 64, v);
            ptx::tmem_wait_ld();
            ptx::reg_fence32(v);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              v[4 * i] = __float_as_uint(__uint_as_float(v[4 * i]) * alpha[0]);
              v[4 * i + 1] = __float_as_uint(__uint_as_float(v[4 * i + 1]) * alpha[0]);
              v[4 * i + 2] = __float_as_uint(__uint_as_float(v[4 * i + 2]) * alpha[1]);
              v[4 * i + 3] = __float_as_uint(__uint_as_float(v[4 * i + 3]) * alpha[1]);
            }
            ptx::tmem_st_16x256b_x8(tO + ch * 64, v);
          }
        }
        ptx::tc_fence_after();
        ptx::tmem_st_16x128b_x16(tmem + lane_off + (uint32_t)(C::kTmemP + pb * 64), pk);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(Plan::kPFull + pb));
      }
      if (!ok) break;
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {  // the row's sum over its four threads
        l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 1);
        l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 2);
      }
      if (!(ok = W.wait_warp(bar(Plan::kLEmpty), le_par))) break;
      le_par ^= 1;
      if ((lane & 3) == 0) {
        row_l[ra] = l[0];
        row_l[ra + 8] = l[1];
        row_m[ra] = m[0];
        row_m[ra + 8] = m[1];
      }
      ptx::mbar_arrive(bar(Plan::kLFull));
    }
  } else if (warp < kWarpMma) {
    // ========================================================== epilogue ===
    ptx::setmaxnreg_dec<C::kRegsEpilogue>();
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tO = tmem + lane_off + (uint32_t)C::kTmemO;
    const bool storer = warp == kWarpEpi && lane == 0;
    int n = 0;  // items finished by this CTA
    bool ok = true;
    ItemReader reader;
    while (ok) {
      int item;
      if (!(ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, true, item)) || item < 0) break;
      const WorkItem it = decode_item<1, false, false>(item, p);
      const uint32_t par = (uint32_t)n & 1u;
      if (!(ok = W.wait_warp(bar(Plan::kLFull), par))) break;
      const float l = row_l[r];
      const float m = row_m[r];
      ptx::mbar_arrive(bar(Plan::kLEmpty));
      if (!(ok = W.wait_warp(bar(Plan::kOFull), par))) break;
      ptx::tc_fence_after();
      const float inv = 1.f / l;
      // Stage the normalised tile in this item's Q buffer (its last S completed before O
      // was full), in the SW128 layout of the output tensor map: row r of 64-column chunk
      // k holds 16-byte unit u at unit position u ^ (r & 7).
      const uint32_t stage = sbase + Plan::kQ + (uint32_t)(n & 1) * Plan::kQBytes + r * 128;
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
        const uint32_t chunk = stage + (uint32_t)(ch >> 1) * Plan::kChunkBytes;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const uint32_t u = (uint32_t)((ch & 1) * 4 + w);
          ptx::st_shared_v4(chunk + ((u ^ (uint32_t)(r & 7)) << 4), pk[4 * w], pk[4 * w + 1], pk[4 * w + 2],
                            pk[4 * w + 3]);
        }
      }
      // O is in registers and shared memory: the next item's first P V may overwrite it.
      ptx::tc_fence_before();
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        ptx::mbar_arrive(bar(Plan::kOEmpty));
        ptx::mbar_arrive(bar(Plan::kStaged));
      }
      if (warp == kWarpEpi) {
        bool sok = true;
        if (storer) {
          // Rows past the end of the sequence fall outside the tensor map and are not written.
          sok = W.wait(bar(Plan::kStaged), par);
          if (sok) {
            const uint32_t src = sbase + Plan::kQ + (uint32_t)(n & 1) * Plan::kQBytes;
            for (int cc = 0; cc < D / 64; ++cc)
              ptx::tma_store_4d(&tmO, src + cc * Plan::kChunkBytes, cc * 64, it.s0 + it.m0, it.h, it.tb);
            ptx::bulk_commit_group();
            ptx::bulk_wait_group_read0();
            ptx::mbar_arrive(bar(Plan::kQEmpty + (n & 1)));  // the producer may load a new Q here
          }
        }
        if (!(ok = __shfl_sync(0xffffffffu, sok ? 1 : 0, 0) != 0)) break;  // warp-uniform
      }
      const int row = it.m0 + r;
      if (p.lse != nullptr && row < it.len)
        p.lse[((long long)it.b * p.H + it.h) * p.N + row] = (m + __log2f(l)) * 0.69314718055994531f;
      ++n;
    }
    if (storer) ptx::bulk_wait_group0();  // global writes of the last stores done
    __syncwarp();
  } else {
    ptx::setmaxnreg_dec<C::kRegsOther>();
    if (warp == kWarpMma) {
      // =============================================================== MMA ===
      // Program order over the CTA's stream of tiles: S(0); then for each tile t: S(t + 1)
      // (possibly the next item's first tile), P(t) V(t). The ring fills come in the same
      // order: K(0); K(t + 1), V(t) for each t.
      constexpr uint32_t idS = make_idesc<T>(kBlockM, kBlockN, false);
      constexpr uint32_t idPV = make_idesc<T>(kBlockM, D, true);
      const uint32_t sKV = sbase + Plan::kKV;
      Ring<NS> ring;
      int s_cnt = 0, p_cnt = 0;  // S and P V tiles issued (buffer = count & 1)
      bool ok = true;
      auto acquire = [&]() -> int {
        const int st = ring.stage;
        const uint32_t ph = ring.phase;
        ring.next();
        if (!W.wait_warp(bar(Plan::kKvFull + st), ph)) return -1;
        ptx::tc_fence_after();
        return st;
      };
      // S(t) = Q K(j)^T into S buffer s_cnt & 1; commits Q empty after the item's last S.
      auto issue_S = [&](int qb, bool last_of_item) -> bool {
        const int sb = s_cnt & 1;
        if (s_cnt >= 2 && !W.wait_warp(bar(Plan::kSFree + sb), (uint32_t)((s_cnt >> 1) - 1) & 1u)) return false;
        const int st = acquire();
        if (st < 0) return false;
        const uint32_t sQ = sbase + Plan::kQ + (uint32_t)qb * Plan::kQBytes;
        const uint64_t a0 = make_sdesc_sw128(sQ, 16, 1024);
        const uint64_t b0 = make_sdesc_sw128(sKV + st * Plan::kStageBytes, 16, 1024);
        const uint32_t dS = tmem + (uint32_t)(C::kTmemS + sb * 128);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * Plan::kChunkBytes + (kk & 3) * 32) >> 4;
          ptx::umma_ss_warp(dS, a0 + off, b0 + off, idS, kk > 0 ? 1u : 0u);
        }
        ptx::tc_commit_warp(bar(Plan::kKvEmpty + st));
        ptx::tc_commit_warp(bar(Plan::kSFull + sb));
        if (last_of_item) ptx::tc_commit_warp(bar(Plan::kQEmpty + qb));
        ++s_cnt;
        return true;
      };
      // O (+)= P(t) V(j); the item's first P V waits for the epilogue to drain O.
      auto issue_PV = [&](int n_item, bool first, bool last) -> bool {
        const int pb = p_cnt & 1;
        if (!W.wait_warp(bar(Plan::kPFull + pb), (uint32_t)(p_cnt >> 1) & 1u)) return false;
        if (first && n_item > 0 && !W.wait_warp(bar(Plan::kOEmpty), (uint32_t)(n_item - 1) & 1u)) return false;
        const int st = acquire();
        if (st < 0) return false;
        const uint64_t b0 = make_sdesc_sw128(sKV + st * Plan::kStageBytes, Plan::kChunkBytes, 1024);
        const uint32_t aP = tmem + (uint32_t)(C::kTmemP + pb * 64);
        const uint32_t dO = tmem + (uint32_t)C::kTmemO;
#pragma unroll
        for (int kk = 0; kk < kBlockN / 16; ++kk) {
          const uint32_t boff = (uint32_t)(kk * 16 * 128) >> 4;
          ptx::umma_ts_warp(dO, aP + (uint32_t)(kk * 8), b0 + boff, idPV, (!first || kk > 0) ? 1u : 0u);
        }
        ptx::tc_commit_warp(bar(Plan::kKvEmpty + st));
        ptx::tc_commit_warp(bar(Plan::kPFree + pb));
        if (last) ptx::tc_commit_warp(bar(Plan::kOFull));
        ++p_cnt;
        return true;
      };
      ItemReader reader;
      int item;
      int n = 0;  // items of this CTA
      if ((ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, true, item)) && item >= 0) {
        WorkItem it = decode_item<1, false, false>(item, p);
        ok = W.wait_warp(bar(Plan::kQFull), 0u);
        if (ok) ok = issue_S(0, it.nb[0] == 1);
        while (ok) {
          const int nb = it.nb[0];
          int next = -1;
          WorkItem nx{};
          for (int j = 0; j < nb && ok; ++j) {
            if (j + 1 < nb) {
              ok = issue_S(n & 1, j + 2 == nb);
            } else {
              if (!(ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, true, next))) break;
              if (next >= 0) {
                nx = decode_item<1, false, false>(next, p);
                const int qb = (n + 1) & 1;
                if (!(ok = W.wait_warp(bar(Plan::kQFull + qb), (uint32_t)((n + 1) >> 1) & 1u))) break;
                ok = issue_S(qb, nx.nb[0] == 1);
              }
            }
            if (ok) ok = issue_PV(n, j == 0, j == nb - 1);
          }
          if (!ok || next < 0) break;
          it = nx;
          ++n;
        }
      }
      // Every MMA this warp issued (and their commit arrivals) must land before the CTA
      // releases TMEM and shared memory.
      ptx::tc_commit_warp(bar(Plan::kDrain));
      if (lane == 0) drain_wait(bar(Plan::kDrain), 0, p.timeout_ns, p.status, p.host_flag);
      __syncwarp();
    } else if (warp == kWarpProd) {
      // ====================================================== producer ===
      // Takes item indices from the shared work counter (one fetch ahead), publishes them
      // to the item ring, loads each item's Q into the Q buffer of its parity and streams
      // K/V tiles in the MMA's order. An item is published when the previous item's last
      // K tile has been issued, so the MMA warp can start the next item early.
      if (lane == 0) {
        const uint64_t pol_q = ptx::policy_evict_first();
        const uint64_t pol_kv = ptx::policy_evict_last();
        const uint32_t sKV = sbase + Plan::kKV;
        Ring<NS> ring;
        int fills = 0, q_fills = 0;
        int published = 0;
        bool ok = true;
        int fetched = atomicAdd(p.work_counter, 1);
        auto publish = [&](int& t) -> bool {
          const int slot = published % kItemRing;
          const uint32_t parity = ((uint32_t)(published / kItemRing) & 1u) ^ 1u;
          if (!W.wait(bar(Plan::kItemEmpty + slot), parity)) return false;
          t = fetched < p.num_items ? fetched : -1;
          if (t >= 0) fetched = atomicAdd(p.work_counter, 1);
          items[slot] = t;
          ptx::mbar_arrive(bar(Plan::kItemFull + slot));
          ++published;
          return true;
        };
        auto load_q = [&](const WorkItem& it, int n) -> bool {
          const int qb = n & 1;
          // Buffer qb was last used by item n - 2: its last S and its O staging are done.
          if (n >= 2 && !W.wait(bar(Plan::kQEmpty + qb), (uint32_t)((n >> 1) - 1) & 1u)) return false;
          const uint32_t dst = sbase + Plan::kQ + (uint32_t)qb * Plan::kQBytes;
          ptx::mbar_arrive_expect_tx(bar(Plan::kQFull + qb), (uint32_t)Plan::kQBytes);
          for (int cc = 0; cc < D / 64; ++cc)
            ptx::tma_load_4d(dst + cc * Plan::kChunkBytes, &tmQ, bar(Plan::kQFull + qb), cc * 64,
                             it.s0 + it.m0, it.h, it.tb, pol_q);
          ++q_fills;
          return true;
        };
        auto fill = [&](const CUtensorMap* map, const WorkItem& it, int j) -> bool {
          const int st = ring.stage;
          const uint32_t ph = ring.phase;
          ring.next();
          if (!W.wait(bar(Plan::kKvEmpty + st), ph ^ 1)) return false;
          ptx::mbar_arrive_expect_tx(bar(Plan::kKvFull + st), (uint32_t)Plan::kStageBytes);
          const int hkv = it.h / p.kv_group;  // grouped-query attention: shared K/V head
#pragma unroll
          for (int cc = 0; cc < D / 64; ++cc)
            ptx::tma_load_4d(sKV + st * Plan::kStageBytes + cc * Plan::kChunkBytes, map, bar(Plan::kKvFull + st),
                             cc * 64, it.s0 + j * kBlockN, hkv, it.tb, pol_kv);
          ++fills;
          return true;
        };
        int t = -1;
        int n = 0;
        if ((ok = publish(t)) && t >= 0) {
          WorkItem it = decode_item<1, false, false>(t, p);
          ok = load_q(it, 0) && fill(&tmK, it, 0);
          while (ok) {
            const int nb = it.nb[0];
            int next = -1;
            WorkItem nx{};
            for (int j = 0; j < nb && ok; ++j) {
              if (j + 1 < nb) {
                ok = fill(&tmK, it, j + 1);
              } else if ((ok = publish(next)) && next >= 0) {
                nx = decode_item<1, false, false>(next, p);
                ok = load_q(nx, n + 1) && fill(&tmK, nx, 0);
              }
              if (ok) ok = fill(&tmV, it, j);
            }
            if (!ok || next < 0) break;
            it = nx;
            ++n;
          }
        }
        // Let every load this thread issued land before the CTA exits.
        const int last = fills < NS ? fills : NS;
        for (int k = 0; k < last; ++k) {
          const int f = fills - 1 - k;
          drain_wait(bar(Plan::kKvFull + (f % NS)), (uint32_t)((f / NS) & 1), p.timeout_ns, p.status, p.host_flag);
        }
        for (int k = q_fills > 2 ? q_fills - 2 : 0; k < q_fills; ++k)
          drain_wait(bar(Plan::kQFull + (k & 1)), (uint32_t)(k >> 1) & 1u, p.timeout_ns, p.status, p.host_flag);
      }
      __syncwarp();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

}  // namespace apex
