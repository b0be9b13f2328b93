// Persistent, warp-specialised causal attention forward for sm_100a (B200).
//
// Replaces the Triton kernels `_attn_fwd_plain` / `_attn_fwd_tma` of
// mls-bench_fused_attention/fused_attention.py:8-144 (same math: softmax(QK^T * scale) V
// with an optional causal mask, fp32 accumulation, output in the input dtype), re-designed
// for Blackwell rather than translated:
//
//   * one CTA per SM, looping over work items (b, h, 256-row query block) in a
//     longest-first order grouped by heads so that concurrently running CTAs share K/V in L2
//     (the reference only reverses the m-block order, fused_attention.py:33-36);
//   * warp roles (16 warps):
//       warps 0-3   softmax for query sub-tile 0 (rows m0 .. m0+127)
//       warps 4-7   softmax for query sub-tile 1 (rows m0+128 .. m0+255)
//       warps 8-11  epilogue: O * (1/l) -> bf16/fp16 -> global, and the fp32 logsumexp
//       warp 12     tcgen05.mma issuer (one thread) + TMEM allocation
//       warp 13     TMA producer (one thread): Q once per item, K/V through an NS-stage ring
//       warps 14-15 idle
//   * S = Q K^T and O += P V run on the 5th-generation tensor cores with both
//     accumulators in TMEM; P is written back into S's TMEM columns and fed to the
//     second GEMM straight from TMEM;
//   * the online softmax keeps a stale running max and rescales O only when the
//     row max grows by more than kRescaleLog2 (log2 units). That keeps most of the
//     reference's "rescale-free" speed (fused_attention.py:61-82) without its
//     overflow hazard for large logits.
//
// TMEM map (512 columns x 128 lanes, lane = query row of a sub-tile):
//   [0,128)   S0 / P0 (P0 packed 2 x 16-bit per column in [0,64))
//   [128,256) S1 / P1
//   [256,256+D)     O0
//   [256+D,256+2D)  O1
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "sm100_ptx.cuh"

namespace apex {

constexpr int kBlockM = 128;   // query rows per sub-tile (= TMEM lanes)
constexpr int kBlockN = 128;   // keys per K/V tile
constexpr int kItemRows = 2 * kBlockM;
constexpr int kThreads = 512;
constexpr float kRescaleLog2 = 8.0f;  // rescale O only when the max grows by > 2^8

// Per-thread register budgets after setmaxnreg. setmaxnreg.inc draws on the registers the
// block was launched with (512 threads x 128, from __launch_bounds__(512, 1)); a split whose
// sum exceeds that would block forever, so it is checked at compile time.
constexpr int kRegsSoftmax = 184;   // 2 warpgroups
constexpr int kRegsEpilogue = 80;   // 1 warpgroup
constexpr int kRegsOther = 56;      // MMA, producer, 2 idle warps
static_assert(128 * (2 * kRegsSoftmax + kRegsEpilogue + kRegsOther) <= kThreads * 128,
              "setmaxnreg split exceeds the launch register allocation");

// Device status bits written by the kernel into the library's status word.
constexpr int kStatusWaitTimeout = 1;   // a pipeline wait exceeded its limit
constexpr int kStatusDrainTimeout = 2;  // an in-flight copy/MMA did not land at teardown

struct AttnParams {
  void* o;
  float* lse;        // nullable, contiguous [B, H, N]
  int* status;       // device status word (bitmask of kStatus*)
  long long o_sb, o_sh, o_sn;  // output strides in elements (d stride is 1)
  int B, H, N;
  int num_mblocks;   // ceil(N / 256)
  int num_kblocks;   // ceil(N / 128)
  int num_items;     // B * H * num_mblocks
  int group_heads;   // heads per L2 scheduling group
  float scale_log2;  // sm_scale * log2(e)
  int causal;
  unsigned long long timeout_ns;
};

template <typename T>
struct DType;
template <>
struct DType<__nv_bfloat16> {
  static constexpr uint32_t kUmmaFormat = 1;  // BF16
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);  // a -> low half (lower column index)
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <>
struct DType<__half> {
  static constexpr uint32_t kUmmaFormat = 0;  // F16
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

// UMMA instruction descriptor, kind::f16, fp32 accumulate, dense.
template <typename T>
__host__ __device__ constexpr uint32_t make_idesc(int M, int N, bool b_mn_major) {
  return (1u << 4)                               // D format: F32
         | (DType<T>::kUmmaFormat << 7)          // A format
         | (DType<T>::kUmmaFormat << 10)         // B format
         | ((b_mn_major ? 1u : 0u) << 16)        // B major-ness
         | ((uint32_t)(N >> 3) << 17)            // N / 8
         | ((uint32_t)(M >> 4) << 24);           // M / 16
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand (sm_100 version bits).
__device__ __forceinline__ uint64_t make_sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                     uint32_t sbo_bytes) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Shared-memory plan. A 128-row tile of D columns is stored as D/64 column chunks,
// each 128 rows x 128 bytes with the TMA 128B swizzle (16 KB per chunk).
template <int D, int NS>
struct SmemPlan {
  static constexpr int kChunkBytes = kBlockM * 128;
  static constexpr int kTileBytes = kBlockM * D * 2;
  static constexpr int kQ = 0;
  static constexpr int kKV = kQ + 2 * kTileBytes;
  static constexpr int kBars = kKV + NS * kTileBytes;
  // barrier slots
  static constexpr int kKvFull = 0;
  static constexpr int kKvEmpty = NS;
  static constexpr int kQFull = 2 * NS;
  static constexpr int kQEmpty = 2 * NS + 1;
  static constexpr int kSFull = 2 * NS + 2;    // [2]
  static constexpr int kPFull = 2 * NS + 4;    // [2]
  static constexpr int kOFull = 2 * NS + 6;    // [2]
  static constexpr int kOEmpty = 2 * NS + 8;   // [2]
  static constexpr int kLFull = 2 * NS + 10;   // [2]
  static constexpr int kLEmpty = 2 * NS + 12;  // [2]
  static constexpr int kDrain = 2 * NS + 14;
  static constexpr int kNumBars = 2 * NS + 15;
  static constexpr int kRowStats = (kBars + kNumBars * 8 + 15) / 16 * 16;  // float l[2][128], m[2][128]
  static constexpr int kMisc = kRowStats + 4 * kBlockM * 4;                // tmem base, abort flag
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kDynamicBytes = kBytes + 1024;  // slack for 1 KB alignment
};

struct WorkItem {
  int b, h, m0;
  int nb0, nb1;  // K/V tiles needed by query sub-tile 0 / 1 (0 = sub-tile past the end)
  int nbmax;
  __device__ __forceinline__ int nb(int i) const { return i == 0 ? nb0 : nb1; }
};

__device__ __forceinline__ WorkItem decode_item(int t, const AttnParams& p) {
  const int BH = p.B * p.H;
  const int MB = p.num_mblocks;
  const int G = p.group_heads;
  const int full = BH / G;
  const int per = G * MB;
  int mb, bh;
  if (t < full * per) {
    const int g = t / per;
    const int r = t - g * per;
    mb = MB - 1 - r / G;
    bh = g * G + r % G;
  } else {
    const int rem = BH - full * G;
    const int r = t - full * per;
    mb = MB - 1 - r / rem;
    bh = full * G + r % rem;
  }
  WorkItem it;
  it.b = bh / p.H;
  it.h = bh - it.b * p.H;
  it.m0 = mb * kItemRows;
  auto tiles = [&](int r0) {
    if (r0 >= p.N) return 0;
    return p.causal ? min(p.num_kblocks, r0 / kBlockN + 1) : p.num_kblocks;
  };
  it.nb0 = tiles(it.m0);
  it.nb1 = tiles(it.m0 + kBlockM);
  it.nbmax = max(it.nb0, it.nb1);
  return it;
}

// Bounded mbarrier wait. Returns false when the CTA is aborting: either another role
// gave up already, or this wait exceeded the time limit (then it raises the CTA abort
// flag and the device status bit). Every loop in the kernel is bounded this way so a
// protocol fault ends the kernel with an error status instead of hanging the GPU.
struct Waiter {
  volatile int* abort_flag;
  int* status;
  unsigned long long timeout_ns;

  __device__ __forceinline__ bool wait(uint32_t bar, uint32_t parity) const {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    return wait_slow(bar, parity);
  }

  __device__ __forceinline__ bool wait_slow(uint32_t bar, uint32_t parity) const {
    const uint64_t t0 = ptx::globaltimer_ns();
    while (true) {
#pragma unroll 1
      for (int i = 0; i < 64; ++i)
        if (ptx::mbar_try_wait(bar, parity)) return true;
      if (*abort_flag) return false;
      if (ptx::globaltimer_ns() - t0 > timeout_ns) {
        *abort_flag = 1;
        atomicOr(status, kStatusWaitTimeout);
        return false;
      }
    }
  }
};

// Wait used only while tearing down: ignores the abort flag, still bounded; a miss is
// reported through the status word.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, unsigned long long limit_ns,
                                           int* status) {
  if (ptx::mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = ptx::globaltimer_ns();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (ptx::globaltimer_ns() - t0 > limit_ns) {
      atomicOr(status, kStatusDrainTimeout);
      return;
    }
  }
}

template <int D, typename T, int NS>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ,
                          const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  static_assert(D == 64 || D == 128, "this kernel covers head dims 64 and 128");
  using Plan = SmemPlan<D, NS>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  const uint32_t sbase = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - raw_addr);

  const int warp = __shfl_sync(0xffffffffu, (int)(threadIdx.x >> 5), 0);
  const int lane = (int)(threadIdx.x & 31);

  auto bar = [&](int slot) -> uint32_t { return sbase + Plan::kBars + slot * 8; };
  float* row_l = reinterpret_cast<float*>(smem + Plan::kRowStats);          // [2][128]
  float* row_m = row_l + 2 * kBlockM;                                        // [2][128]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Plan::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Plan::kMisc + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      ptx::mbar_init(bar(Plan::kKvFull + s), 1);
      ptx::mbar_init(bar(Plan::kKvEmpty + s), 1);
    }
    ptx::mbar_init(bar(Plan::kQFull), 1);
    ptx::mbar_init(bar(Plan::kQEmpty), 1);
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(bar(Plan::kSFull + i), 1);
      ptx::mbar_init(bar(Plan::kPFull + i), kBlockM);
      ptx::mbar_init(bar(Plan::kOFull + i), 1);
      ptx::mbar_init(bar(Plan::kOEmpty + i), kBlockM);
      ptx::mbar_init(bar(Plan::kLFull + i), kBlockM);
      ptx::mbar_init(bar(Plan::kLEmpty + i), kBlockM);
    }
    ptx::mbar_init(bar(Plan::kDrain), 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 12) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), 512);
    ptx::tmem_relinquish();
  }
  if (warp == 13 && lane == 0) {
    ptx::prefetch_tmap(&tmQ);
    ptx::prefetch_tmap(&tmK);
    ptx::prefetch_tmap(&tmV);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const Waiter W{abort_flag, p.status, p.timeout_ns};

  if (warp < 8) {
    // =========================================================== softmax ===
    ptx::setmaxnreg_inc<kRegsSoftmax>();
    const int i = warp >> 2;          // sub-tile
    const int quarter = warp & 3;     // TMEM lane quarter
    const int r = quarter * 32 + lane;  // row within the sub-tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_off + (uint32_t)(i * 128);
    const uint32_t tO = tmem + lane_off + (uint32_t)(256 + i * D);
    const float c = p.scale_log2;
    const int kv_last_valid = p.N - (p.num_kblocks - 1) * kBlockN;  // keys in last K tile
    uint32_t s_par = 0, le_par = 1;
    bool ok = true;
    for (int t = blockIdx.x; t < p.num_items && ok; t += gridDim.x) {
      const WorkItem it = decode_item(t, p);
      const int nb = it.nb(i);
      if (nb == 0) continue;
      const int diag = (it.m0 + i * kBlockM) / kBlockN;
      float m = 0.f, l = 0.f;
      for (int j = 0; j < nb; ++j) {
        ok = __all_sync(0xffffffffu, W.wait(bar(Plan::kSFull + i), s_par));
        if (!ok) break;
        s_par ^= 1;
        ptx::tc_fence_after();
        float s[kBlockN];
#pragma unroll
        for (int ch = 0; ch < kBlockN / 32; ++ch) {
          uint32_t v[32];
          ptx::tmem_ld32(tS + ch * 32, v);
#pragma unroll
          for (int e = 0; e < 32; ++e) s[ch * 32 + e] = __uint_as_float(v[e]);
        }
        ptx::tmem_wait_ld();
        if (p.causal) {
          if (j == diag) {
#pragma unroll
            for (int e = 0; e < kBlockN; ++e)
              if (e > r) s[e] = -INFINITY;
          }
        } else if (j == p.num_kblocks - 1 && kv_last_valid < kBlockN) {
#pragma unroll
          for (int e = 0; e < kBlockN; ++e)
            if (e >= kv_last_valid) s[e] = -INFINITY;
        }
        float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
        for (int e = 4; e < kBlockN; e += 4) {
          mx0 = fmaxf(mx0, s[e]);
          mx1 = fmaxf(mx1, s[e + 1]);
          mx2 = fmaxf(mx2, s[e + 2]);
          mx3 = fmaxf(mx3, s[e + 3]);
        }
        const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * c;
        float alpha = 1.f;
        bool resc = false;
        if (j == 0) {
          m = mx;
        } else if (mx > m + kRescaleLog2) {
          alpha = ptx::ex2(m - mx);
          m = mx;
          resc = true;
        }
        l *= alpha;
        const float nm = -m;
        float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t pk[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float p0 = ptx::ex2(fmaf(s[half * 64 + 2 * e], c, nm));
            const float p1 = ptx::ex2(fmaf(s[half * 64 + 2 * e + 1], c, nm));
            sum0 += p0;
            sum1 += p1;
            pk[e] = DType<T>::pack(p0, p1);
          }
          ptx::tmem_st32(tS + half * 32, pk);
        }
        l += sum0 + sum1;
        if (__any_sync(0xffffffffu, resc)) {
          // Done after S is dead to keep register pressure low. O is quiescent here:
          // the previous P.V of this sub-tile completed before this S tile was
          // signalled, and the next one waits for our P.
#pragma unroll
          for (int ch = 0; ch < D / 32; ++ch) {
            uint32_t v[32];
            ptx::tmem_ld32(tO + ch * 32, v);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
            ptx::tmem_st32(tO + ch * 32, v);
          }
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(Plan::kPFull + i));
      }
      if (!ok) break;
      ok = __all_sync(0xffffffffu, W.wait(bar(Plan::kLEmpty + i), le_par));
      if (!ok) break;
      le_par ^= 1;
      row_l[i * kBlockM + r] = l;
      row_m[i * kBlockM + r] = m;
      ptx::mbar_arrive(bar(Plan::kLFull + i));
    }
  } else if (warp < 12) {
    // ========================================================== epilogue ===
    ptx::setmaxnreg_dec<kRegsEpilogue>();
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint32_t lf_par = 0, of_par = 0;  // bit i: barrier parity for sub-tile i
    auto finish = [&](const WorkItem& it, const int i) -> bool {
      if (!__all_sync(0xffffffffu, W.wait(bar(Plan::kLFull + i), (lf_par >> i) & 1u))) return false;
      lf_par ^= 1u << i;
      const float l = row_l[i * kBlockM + r];
      const float m = row_m[i * kBlockM + r];
      ptx::mbar_arrive(bar(Plan::kLEmpty + i));
      if (!__all_sync(0xffffffffu, W.wait(bar(Plan::kOFull + i), (of_par >> i) & 1u))) return false;
      of_par ^= 1u << i;
      ptx::tc_fence_after();
      const float inv = 1.f / l;
      const int row = it.m0 + i * kBlockM + r;
      const bool valid = row < p.N;
      T* orow = reinterpret_cast<T*>(p.o) + (long long)it.b * p.o_sb + (long long)it.h * p.o_sh +
                (long long)row * p.o_sn;
      const uint32_t tO = tmem + lane_off + (uint32_t)(256 + i * D);
#pragma unroll
      for (int ch = 0; ch < D / 32; ++ch) {
        uint32_t v[32];
        ptx::tmem_ld32(tO + ch * 32, v);
        ptx::tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          pk[e] = DType<T>::pack(__uint_as_float(v[2 * e]) * inv, __uint_as_float(v[2 * e + 1]) * inv);
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + ch * 32);
#pragma unroll
          for (int w = 0; w < 4; ++w)
            dst[w] = make_uint4(pk[4 * w], pk[4 * w + 1], pk[4 * w + 2], pk[4 * w + 3]);
        }
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar(Plan::kOEmpty + i));
      if (p.lse != nullptr && valid)
        p.lse[((long long)it.b * p.H + it.h) * p.N + row] = (m + __log2f(l)) * 0.69314718055994531f;
      return true;
    };
    bool ok = true;
    for (int t = blockIdx.x; t < p.num_items && ok; t += gridDim.x) {
      const WorkItem it = decode_item(t, p);
      if (it.nb0 > 0) ok = finish(it, 0);
      if (ok && it.nb1 > 0) ok = finish(it, 1);
    }
  } else {
    ptx::setmaxnreg_dec<kRegsOther>();
    if (warp == 12) {
      // =============================================================== MMA ===
      constexpr uint32_t idS = make_idesc<T>(kBlockM, kBlockN, false);
      constexpr uint32_t idPV = make_idesc<T>(kBlockM, D, true);
      const uint32_t sQ = sbase + Plan::kQ;
      const uint32_t sKV = sbase + Plan::kKV;
      int stage = 0;
      uint32_t kv_par = 0, q_par = 0;
      uint32_t p_par = 0, oe_par = 3;  // bit i: barrier parity for sub-tile i
      bool ok = true;
      auto issue_S = [&](int i, int st) {
        const uint64_t a0 = make_sdesc_sw128(sQ + i * Plan::kTileBytes, 16, 1024);
        const uint64_t b0 = make_sdesc_sw128(sKV + st * Plan::kTileBytes, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * Plan::kChunkBytes + (kk & 3) * 32) >> 4;
          ptx::umma_ss(tmem + (uint32_t)(i * 128), a0 + off, b0 + off, idS, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_PV = [&](int i, int st, bool acc) {
        const uint64_t b0 = make_sdesc_sw128(sKV + st * Plan::kTileBytes, Plan::kChunkBytes, 1024);
#pragma unroll
        for (int kk = 0; kk < kBlockN / 16; ++kk) {
          const uint32_t off = (uint32_t)(kk * 16 * 128) >> 4;
          ptx::umma_ts(tmem + (uint32_t)(256 + i * D), tmem + (uint32_t)(i * 128 + kk * 8), b0 + off,
                       idPV, (acc || kk > 0) ? 1u : 0u);
        }
      };
      auto next_stage = [&]() {
        if (++stage == NS) {
          stage = 0;
          kv_par ^= 1;
        }
      };
      // O_i += P_i V_j once softmax i published P_i (and, on an item's first tile, once
      // the epilogue released O_i).
      auto pv_step = [&](const int i, int j, int nbi, int sV) -> bool {
        if (!__all_sync(0xffffffffu, W.wait(bar(Plan::kPFull + i), (p_par >> i) & 1u))) return false;
        p_par ^= 1u << i;
        if (j == 0) {
          if (!__all_sync(0xffffffffu, W.wait(bar(Plan::kOEmpty + i), (oe_par >> i) & 1u))) return false;
          oe_par ^= 1u << i;
        }
        ptx::tc_fence_after();
        if (lane == 0) {
          issue_PV(i, sV, j > 0);
          if (j == nbi - 1) ptx::tc_commit(bar(Plan::kOFull + i));
        }
        __syncwarp();
        return true;
      };
      // S_i = Q_i K_{j+1}^T; the K tile is acquired by the first sub-tile that needs it.
      auto s_step = [&](const int i, int& sK) -> bool {
        if (sK < 0) {
          sK = stage;
          if (!__all_sync(0xffffffffu, W.wait(bar(Plan::kKvFull + sK), kv_par))) return false;
          next_stage();
          ptx::tc_fence_after();
        }
        if (lane == 0) {
          issue_S(i, sK);
          ptx::tc_commit(bar(Plan::kSFull + i));
        }
        __syncwarp();
        return true;
      };
      for (int t = blockIdx.x; t < p.num_items && ok; t += gridDim.x) {
        const WorkItem it = decode_item(t, p);
        ok = __all_sync(0xffffffffu, W.wait(bar(Plan::kQFull), q_par));
        if (!ok) break;
        q_par ^= 1;
        int sK = -1;
        if (it.nb0 > 0) ok = s_step(0, sK);
        if (ok && it.nb1 > 0) ok = s_step(1, sK);
        if (!ok) break;
        if (lane == 0) {
          ptx::tc_commit(bar(Plan::kKvEmpty + sK));
          if (it.nbmax == 1) ptx::tc_commit(bar(Plan::kQEmpty));
        }
        __syncwarp();
        for (int j = 0; j < it.nbmax && ok; ++j) {
          const int sV = stage;
          ok = __all_sync(0xffffffffu, W.wait(bar(Plan::kKvFull + sV), kv_par));
          if (!ok) break;
          next_stage();
          sK = -1;
          if (j < it.nb0) ok = pv_step(0, j, it.nb0, sV);
          if (ok && j + 1 < it.nb0) ok = s_step(0, sK);
          if (ok && j < it.nb1) ok = pv_step(1, j, it.nb1, sV);
          if (ok && j + 1 < it.nb1) ok = s_step(1, sK);
          if (!ok) break;
          if (lane == 0) {
            ptx::tc_commit(bar(Plan::kKvEmpty + sV));
            if (sK >= 0) {
              ptx::tc_commit(bar(Plan::kKvEmpty + sK));
              if (j + 2 == it.nbmax) ptx::tc_commit(bar(Plan::kQEmpty));
            }
          }
          __syncwarp();
        }
      }
      // All MMAs issued by this thread (and their commit arrivals) must land before the
      // CTA releases TMEM and shared memory.
      if (lane == 0) {
        ptx::tc_commit(bar(Plan::kDrain));
        drain_wait(bar(Plan::kDrain), 0, p.timeout_ns, p.status);
      }
      __syncwarp();
    } else if (warp == 13) {
      // ========================================================= producer ===
      if (lane == 0) {
        const uint64_t pol_q = ptx::policy_evict_first();
        const uint64_t pol_kv = ptx::policy_evict_last();
        const uint32_t sQ = sbase + Plan::kQ;
        const uint32_t sKV = sbase + Plan::kKV;
        int stage = 0;
        uint32_t kv_par = 0, qe_par = 1;
        int fills = 0;  // K/V stage fills issued
        bool q_filled = false;
        bool ok = true;
        for (int t = blockIdx.x; t < p.num_items && ok; t += gridDim.x) {
          const WorkItem it = decode_item(t, p);
          if (!(ok = W.wait(bar(Plan::kQEmpty), qe_par))) break;
          qe_par ^= 1;
          const int nq = (it.nb0 > 0) + (it.nb1 > 0);
          ptx::mbar_arrive_expect_tx(bar(Plan::kQFull), (uint32_t)(nq * Plan::kTileBytes));
          q_filled = true;
          for (int i = 0; i < 2; ++i) {
            if (it.nb(i) == 0) continue;
            for (int cc = 0; cc < D / 64; ++cc)
              ptx::tma_load_4d(sQ + i * Plan::kTileBytes + cc * Plan::kChunkBytes, &tmQ,
                               bar(Plan::kQFull), cc * 64, it.m0 + i * kBlockM, it.h, it.b, pol_q);
          }
          for (int j = 0; j < it.nbmax && ok; ++j) {
            for (int kv = 0; kv < 2; ++kv) {
              if (!(ok = W.wait(bar(Plan::kKvEmpty + stage), kv_par ^ 1))) break;
              ptx::mbar_arrive_expect_tx(bar(Plan::kKvFull + stage), (uint32_t)Plan::kTileBytes);
              for (int cc = 0; cc < D / 64; ++cc)
                ptx::tma_load_4d(sKV + stage * Plan::kTileBytes + cc * Plan::kChunkBytes,
                                 kv ? (const void*)&tmV : (const void*)&tmK, bar(Plan::kKvFull + stage),
                                 cc * 64, j * kBlockN, it.h, it.b, pol_kv);
              ++fills;
              if (++stage == NS) {
                stage = 0;
                kv_par ^= 1;
              }
            }
          }
        }
        // Let every load this thread issued land before the CTA exits (normally they
        // were all consumed already and these waits return at once).
        const int last = fills < NS ? fills : NS;
        for (int k = 0; k < last; ++k) {
          const int f = fills - 1 - k;  // fill index
          drain_wait(bar(Plan::kKvFull + (f % NS)), (uint32_t)((f / NS) & 1), p.timeout_ns, p.status);
        }
        // qe_par equals the parity of the last Q fill's phase (it flips once per fill).
        if (q_filled) drain_wait(bar(Plan::kQFull), qe_par, p.timeout_ns, p.status);
      }
      __syncwarp();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 12) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

}  // namespace apex
