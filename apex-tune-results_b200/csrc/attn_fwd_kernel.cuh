// Persistent, warp-specialised causal attention forward for sm_100a (B200).
//
// Replaces the Triton kernels `_attn_fwd_plain` / `_attn_fwd_tma` of
// mls-bench_fused_attention/fused_attention.py:8-144 (same math: softmax(QK^T * scale) V
// with an optional causal mask, fp32 accumulation, output in the input dtype), re-designed
// for Blackwell rather than translated:
//
//   * one CTA per SM, looping over work items (b, h, query block of kSub x 128 rows) in a
//     longest-first order grouped by heads so that concurrently running CTAs share K/V in
//     L2 (the reference only reverses the m-block order, fused_attention.py:33-36);
//   * S = Q K^T and O += P V run on the 5th-generation tensor cores (tcgen05.mma) with both
//     accumulators in TMEM;
//   * P never aliases S: it has its own buffer (TMEM columns for d = 64 and 256, shared
//     memory for d = 128, where S and O fill all 512 TMEM columns). So the next S of a
//     query sub-tile is issued as soon as its softmax warps have read the current S into
//     registers, and the softmax warps run back to back instead of waiting for P.V and
//     the next S after every tile;
//   * one MMA-issuing warp per query sub-tile, each walking the shared K/V ring;
//   * the online softmax keeps a stale running max and rescales O only when a row max
//     grows by more than kRescaleLog2 (log2 units). That keeps most of the reference's
//     "rescale-free" speed (fused_attention.py:61-82) without its overflow hazard for large
//     logits.
//
// Warp roles (kSub = 2: d = 64, 128; kSub = 1: d = 256; kCS softmax warpgroups per
// sub-tile, see Cfg):
//   warps [0, 4 kSub kCS)       softmax: kCS warpgroups per query sub-tile; with kCS = 2
//                               unwindowed launches split the sub-tile's rows between them
//                               (16-lane TMEM shapes), windowed d = 64 ones its key columns
//   next 4 warps                epilogue: O * (1/l) -> bf16/fp16 -> global, fp32 logsumexp
//   next kSub warps             tcgen05.mma issuers (warp of sub-tile i; the first also
//                               allocates TMEM)
//   next kSub warps             TMA producers: Q of sub-tile i; the first also fills the
//                               K/V ring
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "sm100_ptx.cuh"

namespace apex {

constexpr int kBlockM = 128;   // query rows per sub-tile (= TMEM lanes)
constexpr int kBlockN = 128;   // keys per K/V tile
constexpr float kRescaleLog2 = 8.0f;  // rescale O only when the max grows by > 2^8

// Device status bits written by the kernel into the library's status word.
constexpr int kStatusWaitTimeout = 1;   // a pipeline wait exceeded its limit
constexpr int kStatusDrainTimeout = 2;  // an in-flight copy/MMA did not land at teardown
constexpr int kStatusSmemAlign = 4;     // dynamic shared memory not 1 KB aligned (not run)

struct AttnParams {
  void* o;
  float* lse;        // nullable, contiguous [B, H, N]
  int* status;       // device status word (bitmask of kStatus*)
  int* host_flag;    // nullable: mapped pinned host word set to 1 with any status bit
  long long o_sb, o_sh, o_sn;  // output strides in elements (d stride is 1)
  int B, H, N;
  int num_mblocks;   // ceil(N / item rows)
  int num_kblocks;   // ceil(N / 128)
  int num_items;     // B * H * num_mblocks
  int group_q;       // L2 scheduling groups hold group_q or group_q + 1 heads ...
  int group_big;     // ... the first group_big groups hold group_q + 1
  int* work_counter; // zeroed before the launch; CTAs take item indices from it
  float scale_log2;  // sm_scale * log2(e)
  int causal;
  int kv_group;      // query heads per K/V head (grouped-query attention; 1 = plain)
  int window;        // causal sliding window: key j visible to row i iff i - window <= j (-1: none)
  // Packed variable-length batch (VAR kernels only): sequence b occupies rows
  // [cu_seqlens[b], cu_seqlens[b + 1]) of tensors with `total` rows; N is the longest
  // sequence. Offsets are clamped to [0, total] and lengths to N in the kernel, so a
  // malformed array cannot move a load or store out of bounds.
  const int* cu_seqlens;
  int total;
  unsigned long long timeout_ns;
};

// Per-head-dim configuration (replaces _CONFIGS, fused_attention.py:148-152).
#ifndef APEX_FWD_CS64
#define APEX_FWD_CS64 2
#endif
// Row-split softmax at d = 128 too: two warpgroups per sub-tile, so four softmax warps share
// each SM sub-partition and overlap one another's exponential phases. P goes to the shared-
// memory P tile with stmatrix (the 16-lane TMEM fragment is the stmatrix fragment). On:
// C3 +1-3.5 % and the fp16 MLS d=128 shape +1-10 % over one warpgroup per sub-tile
// (alternating builds, both orders). With 4-byte P stores instead of stmatrix it measured
// level.
#ifndef APEX_FWD_ROWSPLIT128
#define APEX_FWD_ROWSPLIT128 1
#endif
// The row split at d = 256 too (one sub-tile per CTA: two softmax warpgroups instead of one,
// 512 threads). On: C4 +1.2 % (four alternating pairs, C4 timed alone); all forward tests pass.
#ifndef APEX_FWD_ROWSPLIT256
#define APEX_FWD_ROWSPLIT256 1
#endif

// d = 128: P written into TMEM over the first 64 columns of its own S (instead of a shared-
// memory P buffer). Each sub-tile's next S then waits for its P V, and the freed 64 KB of
// shared memory take the K/V ring from 3 to 5 stages. Off: correct, but measured 18-25 %
// slower (C3 969-985 vs 1179-1215 TFLOP/s): with one MMA warp per sub-tile the two
// sub-tiles fall into step, each softmax idling while its P V and next S run.
#ifndef APEX_FWD_PALIAS128
#define APEX_FWD_PALIAS128 0
#endif

// WIN: the configuration of windowed launches (see kCS).
template <int D, bool WIN = false>
struct Cfg {
  static_assert(D == 64 || D == 128 || D == 256, "head dims 64, 128, 256");
  static constexpr int kSub = D == 256 ? 1 : 2;          // 128-row query sub-tiles per item
  // Softmax warpgroups per sub-tile. Two per sub-tile put more softmax warps on every SM
  // sub-partition (four at d = 64 and 128), so one warp's loads, row max and P store overlap
  // another's exponentials. Unwindowed launches split the sub-tile's rows between the two
  // (kRowSplit: 16-lane TMEM shapes, nothing exchanged; all three head dims). Windowed
  // d = 64 launches split its key columns instead, with the row max exchanged through
  // shared memory and the row sums added in the epilogue (the per-row window bounds do not
  // fit the row split's register budget). The key split needs P in TMEM, so windowed
  // d = 128 and d = 256 launches keep one warpgroup per sub-tile.
  static constexpr int kCS = D == 64 ? APEX_FWD_CS64
                            : ((!WIN && ((D == 128 && APEX_FWD_ROWSPLIT128) || (D == 256 && APEX_FWD_ROWSPLIT256))) ? 2 : 1);
  static constexpr bool kRowSplit = kCS == 2 && !WIN;
  static constexpr int kLSlots = kCS == 2 && !kRowSplit ? 2 : 1;  // row-sum slots per sub-tile
  static constexpr bool kPAlias = D == 128 && APEX_FWD_PALIAS128;  // P over S (see above)
  static constexpr bool kPInTmem = D != 128 || kPAlias;  // else P lives in shared memory
  static constexpr int kParts = D == 256 ? 2 : 1;        // ring stages per K or V tile
  static constexpr int kStageCols = D / kParts;          // head-dim columns per stage
  static constexpr int kNS = D == 64 ? 8 : (D == 128 ? (kPAlias ? 5 : 3) : 5);  // ring stages
  static constexpr int kThreads = 128 * (kSub * kCS + 2);
  static constexpr int kItemRows = kSub * kBlockM;
  // TMEM columns: S_i at i*128; O_i at kTmemO + i*D; P_i at kTmemP + i*kPStride (TMEM
  // variants; with kPAlias, P_i is S_i's first 64 columns).
  static constexpr int kTmemO = 256;
  static constexpr int kTmemP = D == 64 ? 384 : (kPAlias ? 0 : 128);
  static constexpr int kPStride = kPAlias ? 128 : 64;
  // setmaxnreg budgets (multiples of 8): softmax, epilogue, the remaining warpgroup. Their
  // sum x 128 must not exceed the launch allocation (kThreads x (65536 / kThreads)), or
  // setmaxnreg.inc would wait forever; checked below.
  static constexpr int kRegsSoftmax = kCS == 2 ? (D == 128 ? 96 : (D == 256 ? 160 : 88)) : (kSub == 2 ? 184 : 240);
  static constexpr int kRegsEpilogue = kCS == 2 ? (D == 128 ? 56 : (D == 256 ? 96 : 64)) : (kSub == 2 ? 80 : 128);
  static constexpr int kRegsOther = kCS == 2 ? (D == 128 ? 40 : (D == 256 ? 96 : 48)) : (kSub == 2 ? 56 : 136);
  static constexpr int kLaunchRegs = (65536 / kThreads) / 8 * 8;
  static_assert(128 * (kSub * kCS * kRegsSoftmax + kRegsEpilogue + kRegsOther) <= kThreads * kLaunchRegs,
                "setmaxnreg split exceeds the launch register allocation");
  static_assert(kCS == 1 || kPInTmem || kRowSplit, "split softmax columns need P in TMEM");
  static_assert(kTmemO + kSub * D <= 512, "TMEM plan overflows 512 columns");
  static_assert(!kPInTmem || kTmemP + kSub * kPStride <= kTmemO || kTmemP >= kTmemO + kSub * D,
                "P columns overlap O");
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
__host__ __device__ constexpr uint32_t make_idesc(int M, int N, bool b_mn_major, bool a_mn_major = false) {
  return (1u << 4)                               // D format: F32
         | (DType<T>::kUmmaFormat << 7)          // A format
         | (DType<T>::kUmmaFormat << 10)         // B format
         | ((a_mn_major ? 1u : 0u) << 15)        // A major-ness (shared-memory A only)
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

// Shared-memory plan. A 128-row tile of C columns is stored as C/64 column chunks, each
// 128 rows x 128 bytes with the 128-byte swizzle (16 KB per chunk): the layout the TMA
// writes and tcgen05.mma reads for K-major operands. The 1 KB-aligned tile region comes
// first; barriers and row statistics follow it.
// Work items travel from the scheduling producer to every other role through a ring of
// kItemRing slots in shared memory.
constexpr int kItemRing = 4;

template <int D, bool WIN = false>
struct SmemPlan {
  using C = Cfg<D, WIN>;
  static constexpr int kChunkBytes = kBlockM * 128;
  static constexpr int kQTileBytes = kBlockM * D * 2;                 // one sub-tile
  static constexpr int kStageBytes = kBlockN * C::kStageCols * 2;
  static constexpr int kPTileBytes = kBlockM * kBlockN * 2;           // one sub-tile
  static constexpr int kQ = 0;
  static constexpr int kP = kQ + C::kSub * kQTileBytes;
  static constexpr int kKV = kP + (C::kPInTmem ? 0 : C::kSub * kPTileBytes);
  static constexpr int kBars = kKV + C::kNS * kStageBytes;
  // barrier slots
  static constexpr int NS = C::kNS, S = C::kSub;
  static constexpr int kKvFull = 0;
  static constexpr int kKvEmpty = NS;
  static constexpr int kQFull = 2 * NS;
  static constexpr int kQEmpty = kQFull + S;
  static constexpr int kSFull = kQEmpty + S;
  static constexpr int kSFree = kSFull + S;
  static constexpr int kPFull = kSFree + S;
  static constexpr int kPFree = kPFull + S;
  static constexpr int kOFull = kPFree + S;
  static constexpr int kOEmpty = kOFull + S;
  static constexpr int kLFull = kOEmpty + S;
  static constexpr int kLEmpty = kLFull + S;
  static constexpr int kDrain = kLEmpty + S;
  static constexpr int kMaxX = kDrain + S;              // [S * kCS] row-max exchange (kCS = 2)
  static constexpr int kItemFull = kMaxX + S * C::kCS;  // [kItemRing]
  static constexpr int kItemEmpty = kItemFull + kItemRing;  // [kItemRing]
  static constexpr int kNumBars = kItemEmpty + kItemRing;
  // float l[S * kLSlots][128] (row sums, or partial sums of the key halves), m[S][128];
  // then, for the key-column split, the row-max exchange float x[S][kCS][2 tiles][128].
  static constexpr int kRowStats = (kBars + kNumBars * 8 + 15) / 16 * 16;
  static constexpr int kXch = kRowStats + (C::kLSlots + 1) * S * kBlockM * 4;
  static constexpr int kItems = kXch + (C::kCS == 2 && !C::kRowSplit ? S * 2 * 2 * kBlockM * 4 : 0);  // int item[kItemRing]
  static constexpr int kMisc = kItems + kItemRing * 4;                      // tmem base, abort flag
  static constexpr int kBytes = kMisc + 16;
  static constexpr int kMaxDynamic = 232448;  // 227 KB per CTA on sm_100
  // Request 1 KB of alignment slack when it fits; otherwise the kernel relies on the
  // dynamic shared memory base being 1 KB aligned and checks it.
  static constexpr int kDynamicBytes = kBytes + 1024 <= kMaxDynamic ? kBytes + 1024 : kBytes;
  static_assert(kBytes <= kMaxDynamic, "shared-memory plan exceeds 227 KB");
};

struct WorkItem {
  int b, h, m0;
  int s0, len;  // first row of the item's sequence in the tensors, and its length
  int tb;       // batch coordinate of the TMA maps (b; 0 for a packed batch)
  int nkb;      // K/V tiles of the sequence, ceil(len / 128)
  // Query sub-tile i reads K/V tiles [lo[i], nb[i]); nb[i] = 0: sub-tile past the end.
  int lo[2], nb[2];
  int jlo, nbmax;  // K/V tiles of the item: [jlo, nbmax), the union over its sub-tiles
  // Runtime-indexed access without a local-memory copy of the arrays.
  __device__ __forceinline__ int nbi(int i) const { return i == 0 ? nb[0] : nb[1]; }
  __device__ __forceinline__ int loi(int i) const { return i == 0 ? lo[0] : lo[1]; }
};

// Item t -> (b, h, query block). Heads are split into L2 groups of group_q or group_q + 1
// heads (sizes differ by at most one, so no small remainder group comes last); within a
// group items run longest first (query block descending), heads interleaved. CTAs take
// items in this order from a shared counter, so long items start early and the small
// ones fill in at the end.
template <int SUB, bool WIN, bool VAR>
__device__ __forceinline__ WorkItem decode_item(int t, const AttnParams& p) {
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
  WorkItem it;
  it.b = bh / p.H;
  it.h = bh - it.b * p.H;
  it.m0 = mb * SUB * kBlockM;
  if (VAR) {
    const int a = min(max(__ldg(p.cu_seqlens + it.b), 0), p.total);
    const int e = min(max(__ldg(p.cu_seqlens + it.b + 1), a), p.total);
    it.s0 = a;
    it.len = min(e - a, p.N);
    it.tb = 0;
    it.nkb = (it.len + kBlockN - 1) / kBlockN;
  } else {
    it.s0 = 0;
    it.len = p.N;
    it.tb = it.b;
    it.nkb = p.num_kblocks;
  }
  auto tiles = [&](int r0) {
    if (r0 >= it.len) return 0;
    return p.causal ? min(it.nkb, r0 / kBlockN + 1) : it.nkb;
  };
  // First K/V tile a sub-tile starting at row r0 can see: with a sliding window, row r0
  // sees keys >= r0 - window (later rows see fewer low keys, masked per element).
  auto first = [&](int r0) { return WIN ? max(0, r0 - p.window) / kBlockN : 0; };
  it.nb[0] = tiles(it.m0);
  it.nb[1] = SUB == 2 ? tiles(it.m0 + kBlockM) : 0;
  it.lo[0] = first(it.m0);
  it.lo[1] = SUB == 2 ? first(it.m0 + kBlockM) : 0;
  it.nbmax = max(it.nb[0], it.nb[1]);
  it.jlo = it.lo[0];  // lo[1] >= lo[0] whenever sub-tile 1 has tiles
  return it;
}

// exp2 on the FMA pipe for a pair of exponents x <= ~9 (-inf never reaches it).
// Cody-Waite style split x = j + f with j = rint(x) (1.5*2^23 rounding constant) and
// f = x - j in [-1/2, 1/2] (both exact); 2^f from a degree-3 polynomial with c0 = 1 whose
// coefficients minimise the maximum relative error on [-1/2, 1/2] (fitted for this
// kernel by linear programming: 1.0e-4, far below the bf16/fp16 rounding of P; x = 0
// gives exactly 1); 2^j is added into the exponent bits. x is clamped at -125 so the
// result stays a normal float.
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23
constexpr float kExp2C1 = 0.69328290224f;
constexpr float kExp2C2 = 0.24221095443f;
constexpr float kExp2C3 = 0.05500892922f;

__device__ __forceinline__ float2 exp2_poly_pair(float2 x) {
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 t = __fadd2_rn(x, make_float2(kRoundMagic, kRoundMagic));    // MAGIC + j
  const float2 jf = __fadd2_rn(t, make_float2(-kRoundMagic, -kRoundMagic));  // j, exact
  const float2 f = __fadd2_rn(x, make_float2(-jf.x, -jf.y));                 // x - j, exact
  float2 pl = __ffma2_rn(make_float2(kExp2C3, kExp2C3), f, make_float2(kExp2C2, kExp2C2));
  pl = __ffma2_rn(pl, f, make_float2(kExp2C1, kExp2C1));
  pl = __ffma2_rn(pl, f, make_float2(1.f, 1.f));
  const int ex = __float_as_int(t.x) << 23;  // j << 23 (the 1.5*2^23 offset shifts out)
  const int ey = __float_as_int(t.y) << 23;
  return make_float2(__int_as_float(__float_as_int(pl.x) + ex), __int_as_float(__float_as_int(pl.y) + ey));
}

// Records a device-side error: the bit goes into the device status word, and a nonzero
// word into the caller's mapped pinned host flag (when there is one), which the host entry
// points read before every launch so the next call fails instead of returning quietly.
__device__ __forceinline__ void report_error(int* status, int* host_flag, int bit) {
  atomicOr(status, bit);
  if (host_flag != nullptr) {
    *reinterpret_cast<volatile int*>(host_flag) = 1;
    __threadfence_system();
  }
}

// Bounded mbarrier wait. Returns false when the CTA is aborting: either another role
// gave up already, or this wait exceeded the time limit (then it raises the CTA abort
// flag and the device status bit). Every loop in the kernel is bounded this way so a
// protocol fault ends the kernel with an error status instead of hanging the GPU.
struct Waiter {
  volatile int* abort_flag;
  int* status;
  unsigned long long timeout_ns;
  int* host_flag;

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
        report_error(status, host_flag, kStatusWaitTimeout);
        return false;
      }
    }
  }

  // Whole-warp form: every lane waits, the result is warp-uniform.
  __device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity) const {
    return __all_sync(0xffffffffu, wait(bar, parity));
  }
};

// Wait used only while tearing down: ignores the abort flag, still bounded; a miss is
// reported through the status word.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, unsigned long long limit_ns,
                                           int* status, int* host_flag) {
  if (ptx::mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = ptx::globaltimer_ns();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (ptx::globaltimer_ns() - t0 > limit_ns) {
      report_error(status, host_flag, kStatusDrainTimeout);
      return;
    }
  }
}

// Position in the K/V ring, as every consumer and the producer walk it. Per item the
// fills are K(0); then for j = 0 .. nbmax-1: K(j+1) (if j+1 < nbmax), V(j); each K or V
// tile takes kParts consecutive stages. K runs one tile ahead of V because S(j+1) is
// issued at the start of softmax(j) while P(j) V(j) waits for its end. With kPAlias the
// order is V(j), then K(j+1): S(j+1) overwrites P(j), so it follows P(j) V(j).
template <int NS>
struct Ring {
  int stage = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next() {
    if (++stage == NS) {
      stage = 0;
      phase ^= 1;
    }
  }
};

// Reader side of the item ring: every role walks the same sequence of item indices that
// the scheduling producer publishes; index -1 ends the sequence. Each reading warp releases
// a slot once (lane 0) after reading it.
struct ItemReader {
  int k = 0;
  __device__ __forceinline__ bool next(const Waiter& W, uint32_t full0, uint32_t empty0,
                                       const int* items, bool whole_warp, int& t) {
    const int slot = k % kItemRing;
    const uint32_t parity = (uint32_t)(k / kItemRing) & 1u;
    ++k;
    if (whole_warp) {
      if (!W.wait_warp(full0 + slot * 8, parity)) return false;
      t = items[slot];
      __syncwarp();
      if ((threadIdx.x & 31) == 0) ptx::mbar_arrive(empty0 + slot * 8);
    } else {
      if (!W.wait(full0 + slot * 8, parity)) return false;
      t = items[slot];
      ptx::mbar_arrive(empty0 + slot * 8);
    }
    return true;
  }
};

// EMU8: of every 8 column pairs of an unmasked S tile, how many take exp2 from the
// FMA-pipe polynomial instead of MUFU (0 = all MUFU).
// WIN: the launch uses a causal sliding window (p.window >= 0); without it the window
// logic compiles away. VAR: packed variable-length batch (p.cu_seqlens).
template <int D, typename T, int EMU8, bool WIN, bool VAR>
__global__ void __launch_bounds__(Cfg<D, WIN>::kThreads, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ,
                          const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using C = Cfg<D, WIN>;
  using Plan = SmemPlan<D, WIN>;
  constexpr int SUB = C::kSub;
  constexpr int NS = C::kNS;
  constexpr int KP = C::kParts;
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
  constexpr int CS = C::kCS;
  constexpr int kWarpEpi = 4 * SUB * CS;  // first epilogue warp
  constexpr int kWarpMma = kWarpEpi + 4;  // first MMA warp
  constexpr int kWarpProd = kWarpMma + SUB;

  auto bar = [&](int slot) -> uint32_t { return sbase + Plan::kBars + slot * 8; };
  float* row_l = reinterpret_cast<float*>(smem + Plan::kRowStats);   // [SUB * kLSlots][128]
  float* row_m = row_l + SUB * C::kLSlots * kBlockM;                  // [SUB][128]
  int* items = reinterpret_cast<int*>(smem + Plan::kItems);           // [kItemRing]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Plan::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Plan::kMisc + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      ptx::mbar_init(bar(Plan::kKvFull + s), 1);
      ptx::mbar_init(bar(Plan::kKvEmpty + s), SUB);  // one release per MMA warp
    }
    for (int i = 0; i < SUB; ++i) {
      ptx::mbar_init(bar(Plan::kQFull + i), 1);
      ptx::mbar_init(bar(Plan::kQEmpty + i), 1);
      ptx::mbar_init(bar(Plan::kSFull + i), 1);
      ptx::mbar_init(bar(Plan::kSFree + i), kBlockM * CS);
      ptx::mbar_init(bar(Plan::kPFull + i), kBlockM * CS);
      ptx::mbar_init(bar(Plan::kPFree + i), 1);
      ptx::mbar_init(bar(Plan::kOFull + i), 1);
      ptx::mbar_init(bar(Plan::kOEmpty + i), kBlockM);
      ptx::mbar_init(bar(Plan::kLFull + i), kBlockM * CS);
      ptx::mbar_init(bar(Plan::kLEmpty + i), kBlockM);
      ptx::mbar_init(bar(Plan::kDrain + i), 1);
      for (int h = 0; h < CS; ++h) ptx::mbar_init(bar(Plan::kMaxX + i * CS + h), kBlockM);
    }
    // Readers of the item ring: softmax, epilogue and MMA warps, and the Q producer of
    // sub-tile 1 (the ring producer writes it).
    constexpr int kItemReaders = 4 * SUB * CS + 4 + SUB + (SUB - 1);
    for (int k = 0; k < kItemRing; ++k) {
      ptx::mbar_init(bar(Plan::kItemFull + k), 1);
      ptx::mbar_init(bar(Plan::kItemEmpty + k), kItemReaders);
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
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const Waiter W{abort_flag, p.status, p.timeout_ns, p.host_flag};

  if (warp < kWarpEpi) {
    // =========================================================== softmax ===
    ptx::setmaxnreg_inc<C::kRegsSoftmax>();
    if constexpr (C::kRowSplit) {
      // Two warpgroups per sub-tile split its rows: in each 32-lane TMEM quarter, the warp
      // of warpgroup h takes lanes 16h .. 16h + 15 (16-lane tcgen05.ld/st shapes), all 128
      // keys of the tile. Thread t holds rows ra = lb + t/4 and ra + 8, keys 8e + kq + {0,1}
      // (e = 0..15, kq = 2 (t % 4)); the four threads of a row reduce its max with two
      // shuffles. The warpgroups never exchange anything, so neither waits for the other:
      // C2 and the fp16 MLS d=64 shape +4.5 % over splitting the keys with a per-tile row-max
      // exchange (measured alternating builds). Windowed launches keep the key split below:
      // the per-row window bounds push this form past its 88-register budget (spills,
      // -14 %). P goes to TMEM, or at d = 128 to the sub-tile's shared-memory P buffer.
      const int i = (warp >> 2) >> 1;                     // sub-tile
      const int lb = (warp & 3) * 32 + ((warp >> 2) & 1) * 16;  // first TMEM lane (= row) of this warp
      const int ra = lb + (lane >> 2);
      const int kq = 2 * (lane & 3);
      const uint32_t lane_off = (uint32_t)lb << 16;
      const uint32_t tS = tmem + lane_off + (uint32_t)(i * 128);
      const uint32_t tO = tmem + lane_off + (uint32_t)(C::kTmemO + i * D);
      const uint32_t tP = tmem + lane_off + (uint32_t)(C::kTmemP + i * C::kPStride);
      // P in shared memory (d = 128): the SW128 K-major tile of the sub-tile, keys 0-63 and
      // 64-127 in two 16 KB chunks; 16-byte unit u of row R sits at unit position
      // u ^ (R & 7) (stored with stmatrix below).
      const float c = p.scale_log2;
      const float2 c2 = make_float2(c, c);
      uint32_t s_par = 0, le_par = 1, pf_par = 0;
      // P store addresses (d = 128), fixed per lane: stmatrix instruction k writes 16-byte
      // unit e = 2k + lane / 16 of row R = lb + 8 ((lane / 8) % 2) + lane % 8, so its unit
      // within the 64-key chunk k / 4 is (2 (k % 4) + lane / 16) ^ (R % 8), and R % 8 = lane % 8.
      uint32_t p_row[4];
      {
        const uint32_t sP0 = sbase + Plan::kP + i * Plan::kPTileBytes;
        const uint32_t row = (uint32_t)(lb + 8 * ((lane >> 3) & 1) + (lane & 7));
#pragma unroll
        for (int q = 0; q < 4; ++q)
          p_row[q] = sP0 + row * 128 + (((uint32_t)(2 * q + (lane >> 4)) ^ (uint32_t)(lane & 7)) << 4);
      }
      int p_written = 0;  // P tiles handed over so far (the buffer is reused every tile)
      bool ok = true;
      ItemReader reader;
      while (ok) {
        int t;
        if (!(ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, true, t)) || t < 0) break;
        const WorkItem it = decode_item<SUB, WIN, VAR>(t, p);
        const int nb = it.nbi(i);
        const int lo = it.loi(i);
        if (nb == 0) continue;
        const int r0 = it.m0 + i * kBlockM;  // first row of the sub-tile
        const int diag = r0 / kBlockN;
        float m[2] = {0.f, 0.f}, l[2] = {0.f, 0.f};  // rows ra, ra + 8
        for (int j = lo; j < nb; ++j) {
          if (!(ok = W.wait_warp(bar(Plan::kSFull + i), s_par))) break;
          s_par ^= 1;
          ptx::tc_fence_after();
          // v[h][4i' + 2rr + b] = S(row ra + 8 rr, key 8e + kq + b), e = 8h + i'
          uint32_t v[2][32];
          ptx::tmem_ld_16x256b_x8(tS, v[0]);
          ptx::tmem_ld_16x256b_x8(tS + 64, v[1]);
          ptx::tmem_wait_ld();
          ptx::reg_fence32(v[0]);
          ptx::reg_fence32(v[1]);
          // S is in registers: the MMA warp may overwrite it with the next tile's scores.
          ptx::tc_fence_before();
          ptx::mbar_arrive(bar(Plan::kSFree + i));
          const bool diag_tile = p.causal && j == diag;
          const int kv_last_valid = it.len - (it.nkb - 1) * kBlockN;  // keys in the last K tile
          const bool tail_tile = !p.causal && j == it.nkb - 1 && kv_last_valid < kBlockN;
          const bool masked = diag_tile || tail_tile;  // warp-uniform
          if (masked) {
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
              const int row = ra + 8 * rr;
              const int limit = diag_tile ? row + 1 : kv_last_valid;  // keys >= limit are masked
#pragma unroll
              for (int e = 0; e < 16; ++e)
#pragma unroll
                for (int b = 0; b < 2; ++b)
                  if (8 * e + kq + b >= limit) v[e >> 3][4 * (e & 7) + 2 * rr + b] = __float_as_uint(-INFINITY);
            }
          }
          bool resc = false;
          float alpha[2] = {1.f, 1.f};
          float2 nm2[2];
          // Both rows' max trees and shuffles first, in one branch-free block so that they
          // overlap; the rescale decisions follow (C2 +1.5 %, C3 +3 % over deciding each
          // row right after its own max, measured alternating builds).
          float mxr[2];  // the tile's row maxima, log2 domain
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            float m0 = fmaxf(__uint_as_float(v[0][2 * rr]), __uint_as_float(v[0][2 * rr + 1]));
            float m1 = fmaxf(__uint_as_float(v[1][2 * rr]), __uint_as_float(v[1][2 * rr + 1]));
#pragma unroll
            for (int e = 1; e < 8; ++e) {
              m0 = ptx::fmax3(m0, __uint_as_float(v[0][4 * e + 2 * rr]), __uint_as_float(v[0][4 * e + 2 * rr + 1]));
              m1 = ptx::fmax3(m1, __uint_as_float(v[1][4 * e + 2 * rr]), __uint_as_float(v[1][4 * e + 2 * rr + 1]));
            }
            float mx = fmaxf(m0, m1);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));  // the four threads of the row
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mxr[rr] = mx * c;
          }
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            if (j == lo) {
              m[rr] = mxr[rr];
            } else if (mxr[rr] > m[rr] + kRescaleLog2) {
              alpha[rr] = ptx::ex2(m[rr] - mxr[rr]);
              m[rr] = mxr[rr];
              resc = true;
            }
            l[rr] *= alpha[rr];
            nm2[rr] = make_float2(-m[rr], -m[rr]);
          }
          // p = exp2(s c - m), packed to 16-bit pairs in the 16x128b store layout:
          // pk[2e + rr] = P(row ra + 8 rr, keys 8e + kq, 8e + kq + 1)
          uint32_t pk[32];
          float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
          auto exps = [&](auto poly) {
            constexpr bool kPoly = decltype(poly)::value;
#pragma unroll
            for (int e = 0; e < 16; ++e) {
#pragma unroll
              for (int rr = 0; rr < 2; ++rr) {
                const float2 x = __ffma2_rn(make_float2(__uint_as_float(v[e >> 3][4 * (e & 7) + 2 * rr]),
                                                        __uint_as_float(v[e >> 3][4 * (e & 7) + 2 * rr + 1])),
                                            c2, nm2[rr]);
                float2 pr;
                if (kPoly && ((2 * e + rr) & 7) < EMU8) pr = exp2_poly_pair(x);
                else pr = make_float2(ptx::ex2(x.x), ptx::ex2(x.y));
                acc[rr] = __fadd2_rn(acc[rr], pr);
                pk[2 * e + rr] = DType<T>::pack(pr.x, pr.y);
              }
            }
          };
          if (masked) exps(std::false_type{});  // masked keys hold -inf: MUFU gives exactly 0
          else exps(std::integral_constant<bool, (EMU8 > 0)>{});
          l[0] += acc[0].x + acc[0].y;
          l[1] += acc[1].x + acc[1].y;
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
            for (int ch = 0; ch < D / 64; ++ch) {
              uint32_t o[32];
              ptx::tmem_ld_16x256b_x8(tO + ch * 64, o);
              ptx::tmem_wait_ld();
              ptx::reg_fence32(o);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                o[4 * e] = __float_as_uint(__uint_as_float(o[4 * e]) * alpha[0]);
                o[4 * e + 1] = __float_as_uint(__uint_as_float(o[4 * e + 1]) * alpha[0]);
                o[4 * e + 2] = __float_as_uint(__uint_as_float(o[4 * e + 2]) * alpha[1]);
                o[4 * e + 3] = __float_as_uint(__uint_as_float(o[4 * e + 3]) * alpha[1]);
              }
              ptx::tmem_st_16x256b_x8(tO + ch * 64, o);
            }
          }
          if constexpr (C::kPInTmem) {
            ptx::tmem_st_16x128b_x16(tP, pk);
          } else {
            // pk[m], m = 2e + rr, is this thread's pair of the 8 x 8 block (rows lb + 8rr ..,
            // keys 8e ..) in exactly the stmatrix fragment layout (row lane / 4, columns
            // 2 (lane % 4) ..). Eight stmatrix.x4 store the warp's 16 rows: matrix m of
            // instruction k is 4k + lane / 8, and this lane gives the address of its row
            // lane % 8: p_row[k & 3] in 64-key chunk k / 4 (the immediate offset).
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              ptx::stmatrix_x4<0>(p_row[k], pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
              ptx::stmatrix_x4<Plan::kChunkBytes>(p_row[k], pk[16 + 4 * k], pk[17 + 4 * k], pk[18 + 4 * k],
                                                  pk[19 + 4 * k]);
            }
            ptx::fence_proxy_async_smem();
          }
          ptx::tmem_wait_st();
          ptx::tc_fence_before();
          ptx::mbar_arrive(bar(Plan::kPFull + i));
        }
        if (!ok) break;
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {  // the row's sum over its four threads
          l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 1);
          l[rr] += __shfl_xor_sync(0xffffffffu, l[rr], 2);
        }
        if (!(ok = W.wait_warp(bar(Plan::kLEmpty + i), le_par))) break;
        le_par ^= 1;
        if ((lane & 3) == 0) {
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            row_l[i * kBlockM + ra + 8 * rr] = l[rr];  // one slot per sub-tile: the full row sum
            row_m[i * kBlockM + ra + 8 * rr] = m[rr];
          }
        }
        ptx::mbar_arrive(bar(Plan::kLFull + i));
      }
    } else {
      constexpr int kCols = kBlockN / CS;  // key columns of the tile this warpgroup handles
      constexpr int NH = kCols / 64;       // 64-key halves among them
      const int i = (warp >> 2) / CS;     // sub-tile
      const int cs = (warp >> 2) % CS;    // column part: keys [cs * kCols, (cs + 1) * kCols)
      const int quarter = warp & 3;       // TMEM lane quarter
      const int r = quarter * 32 + lane;  // row within the sub-tile
      const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
      const uint32_t tS = tmem + lane_off + (uint32_t)(i * 128 + cs * kCols);
      const uint32_t tO = tmem + lane_off + (uint32_t)(C::kTmemO + i * D);
      const uint32_t tP = tmem + lane_off + (uint32_t)(C::kTmemP + i * C::kPStride + cs * (kCols / 2));
      float* xch = reinterpret_cast<float*>(smem + Plan::kXch);  // [SUB][CS][2][128]
      int tcount = 0;  // tiles this warpgroup processed (row-max exchange slot and parity)
      // Row r of P in shared memory: two 16 KB chunks (keys 0-63, 64-127) of the SW128
      // K-major layout; 16-byte unit u of the row sits at unit position u ^ (r & 7).
      const uint32_t sP = sbase + Plan::kP + i * Plan::kPTileBytes + r * 128;
      const float c = p.scale_log2;
      const float2 c2 = make_float2(c, c);
      uint32_t s_par = 0, le_par = 1, pf_par = 0;
      int p_written = 0;  // P tiles handed over so far (the buffer is reused every tile)
      bool ok = true;
      ItemReader reader;
      while (ok) {
        int t;
        if (!(ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, true, t)) || t < 0) break;
        const WorkItem it = decode_item<SUB, WIN, VAR>(t, p);
        const int nb = it.nbi(i);
        const int lo = it.loi(i);
        if (nb == 0) continue;
        const int r0 = it.m0 + i * kBlockM;  // first row of the sub-tile
        const int diag = r0 / kBlockN;
        float m = 0.f, l = 0.f;
        for (int j = lo; j < nb; ++j) {
          if (!(ok = W.wait_warp(bar(Plan::kSFull + i), s_par))) break;
          s_par ^= 1;
          ptx::tc_fence_after();
          float s[kCols];
          {
            uint32_t v[kCols / 32][32];
#pragma unroll
            for (int ch = 0; ch < kCols / 32; ++ch) ptx::tmem_ld32(tS + ch * 32, v[ch]);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int ch = 0; ch < kCols / 32; ++ch) {
              ptx::reg_fence32(v[ch]);  // no use of the loaded values above the wait
#pragma unroll
              for (int e = 0; e < 32; ++e) s[ch * 32 + e] = __uint_as_float(v[ch][e]);
            }
          }
          // S is in registers: the MMA warp may overwrite it with the next tile's scores.
          ptx::tc_fence_before();
          ptx::mbar_arrive(bar(Plan::kSFree + i));
          const bool diag_tile = p.causal && j == diag;
          const int kv_last_valid = it.len - (it.nkb - 1) * kBlockN;  // keys in the last K tile
          const bool tail_tile = !p.causal && j == it.nkb - 1 && kv_last_valid < kBlockN;
          // Sliding window: the tile holds keys below some row's window start iff its first
          // key is below the sub-tile's last row minus the window.
          const bool win_tile = WIN && j * kBlockN < r0 + kBlockM - 1 - p.window;
          const bool masked = diag_tile || tail_tile || win_tile;  // warp-uniform
          if (masked) {
            const int kv_limit = diag_tile ? r + 1 : (tail_tile ? kv_last_valid : kBlockN);  // keys >= limit masked
            const int kv_first = win_tile ? r0 + r - p.window - j * kBlockN : 0;            // keys < first masked
#pragma unroll
            for (int e = 0; e < kCols; ++e)
              if (e + cs * kCols >= kv_limit || e + cs * kCols < kv_first) s[e] = -INFINITY;
          }
          float mx0 = fmaxf(s[0], s[1]), mx1 = fmaxf(s[2], s[3]);
          float mx2 = fmaxf(s[4], s[5]), mx3 = fmaxf(s[6], s[7]);
          static_assert(kBlockN % 8 == 0, "row max consumes 8 scores per step");
#pragma unroll
          for (int e = 8; e < kCols; e += 8) {
            mx0 = ptx::fmax3(mx0, s[e], s[e + 1]);
            mx1 = ptx::fmax3(mx1, s[e + 2], s[e + 3]);
            mx2 = ptx::fmax3(mx2, s[e + 4], s[e + 5]);
            mx3 = ptx::fmax3(mx3, s[e + 6], s[e + 7]);
          }
          float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * c;  // log2 domain
          if (CS == 2) {
            // Row max over the whole tile: publish this part's max, take the partner's. Slots
            // alternate by tile; a slot is rewritten two tiles later, after the partner has
            // read it (it reads tile t before it can reach the exchange of tile t + 1).
            const int slot = tcount & 1;
            xch[((i * CS + cs) * 2 + slot) * kBlockM + r] = mx;
            ptx::mbar_arrive(bar(Plan::kMaxX + i * CS + cs));
            if (!(ok = W.wait_warp(bar(Plan::kMaxX + i * CS + (1 - cs)), (uint32_t)slot))) break;
            mx = fmaxf(mx, xch[((i * CS + (1 - cs)) * 2 + slot) * kBlockM + r]);
          }
          ++tcount;
          float alpha = 1.f;
          bool resc = false;
          if (j == lo) {
            m = mx;  // -inf when the window hides this whole tile from the row
          } else if (mx > m + kRescaleLog2) {  // from m = -inf: alpha = 0, as it must be
            alpha = ptx::ex2(m - mx);
            m = mx;
            resc = true;
          }
          l *= alpha;
          // p = exp2(s*c - m), packed to 16-bit pairs: pk[key half][32]
          const float m_use = (WIN && m == -INFINITY) ? 0.f : m;  // all keys masked: p = 0, not NaN
          const float2 nm2 = make_float2(-m_use, -m_use);
          float2 sa = make_float2(0.f, 0.f), sb = make_float2(0.f, 0.f);
          uint32_t pk[NH][32];
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
          for (int h = 0; h < NH; ++h) {
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
            for (int ch = cs * (D / 32 / CS); ch < (cs + 1) * (D / 32 / CS); ++ch) {  // this part's O columns
              uint32_t v[32];
              ptx::tmem_ld32(tO + ch * 32, v);
              ptx::tmem_wait_ld();
              ptx::reg_fence32(v);
#pragma unroll
              for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
              ptx::tmem_st32(tO + ch * 32, v);
            }
          }
          if (C::kPInTmem) {
#pragma unroll
            for (int h = 0; h < NH; ++h) ptx::tmem_st32(tP + h * 32, pk[h]);
            ptx::tmem_wait_st();
          } else {
#pragma unroll
            for (int h = 0; h < NH; ++h)
#pragma unroll
              for (int u = 0; u < 8; ++u)
                ptx::st_shared_v4(sP + h * Plan::kChunkBytes + ((u ^ (r & 7)) << 4), pk[h][4 * u],
                                  pk[h][4 * u + 1], pk[h][4 * u + 2], pk[h][4 * u + 3]);
            ptx::fence_proxy_async_smem();
            ptx::tmem_wait_st();  // the O rescale stores, if any
          }
          ptx::tc_fence_before();
          ptx::mbar_arrive(bar(Plan::kPFull + i));
        }
        if (!ok) break;
        if (!(ok = W.wait_warp(bar(Plan::kLEmpty + i), le_par))) break;
        le_par ^= 1;
        row_l[(i * CS + cs) * kBlockM + r] = l;  // this part's share of the row sum
        if (cs == 0) row_m[i * kBlockM + r] = m;
        ptx::mbar_arrive(bar(Plan::kLFull + i));
      }
    }
  } else if (warp < kWarpMma) {
    // ========================================================== epilogue ===
    ptx::setmaxnreg_dec<C::kRegsEpilogue>();
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint32_t lf_par = 0, of_par = 0;  // bit i: barrier parity for sub-tile i
    auto finish = [&](const WorkItem& it, const int i) -> bool {
      if (!W.wait_warp(bar(Plan::kLFull + i), (lf_par >> i) & 1u)) return false;
      lf_par ^= 1u << i;
      float l = row_l[(i * C::kLSlots) * kBlockM + r];
      if (C::kLSlots == 2) l += row_l[(i * C::kLSlots + 1) * kBlockM + r];
      const float m = row_m[i * kBlockM + r];
      ptx::mbar_arrive(bar(Plan::kLEmpty + i));
      if (!W.wait_warp(bar(Plan::kOFull + i), (of_par >> i) & 1u)) return false;
      of_par ^= 1u << i;
      ptx::tc_fence_after();
      const float inv = 1.f / l;
      const int row = it.m0 + i * kBlockM + r;
      const bool valid = row < it.len;
      T* orow = reinterpret_cast<T*>(p.o) + (long long)it.b * p.o_sb * (VAR ? 0 : 1) +
                (long long)it.h * p.o_sh + (long long)(it.s0 + row) * p.o_sn;
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
          for (int w = 0; w < 4; ++w)
            dst[w] = make_uint4(pk[4 * w], pk[4 * w + 1], pk[4 * w + 2], pk[4 * w + 3]);
        }
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar(Plan::kOEmpty + i));
      if (p.lse != nullptr && valid) {
        // [B, H, N]; packed batch: [H, total]
        const long long li = VAR ? (long long)it.h * p.total + it.s0 + row
                                 : ((long long)it.b * p.H + it.h) * p.N + row;
        p.lse[li] = (m + __log2f(l)) * 0.69314718055994531f;
      }
      return true;
    };
    bool ok = true;
    ItemReader reader;
    while (ok) {
      int t;
      if (!(ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, true, t)) || t < 0) break;
      const WorkItem it = decode_item<SUB, WIN, VAR>(t, p);
      for (int i = 0; i < SUB && ok; ++i)
        if (it.nbi(i) > 0) ok = finish(it, i);
    }
  } else {
    ptx::setmaxnreg_dec<C::kRegsOther>();
    if (warp < kWarpMma + SUB) {
      // =============================================================== MMA ===
      // Warp i issues every MMA of query sub-tile i: S_i(j) = Q_i K(j)^T once softmax i
      // has read S_i(j-1), and O_i += P_i(j) V(j) once softmax i has written P_i(j). The
      // whole warp runs the issue path and elect.sync picks the issuing lane (lane 0), so
      // MMAs and their commits come from one thread.
      const int i = warp - kWarpMma;
      constexpr uint32_t idS = make_idesc<T>(kBlockM, kBlockN, false);
      constexpr uint32_t idPV = make_idesc<T>(kBlockM, C::kStageCols, true);
      const uint32_t sQ = sbase + Plan::kQ + i * Plan::kQTileBytes;
      const uint32_t sKV = sbase + Plan::kKV;
      const uint32_t sPi = sbase + Plan::kP + i * Plan::kPTileBytes;
      const uint32_t tSi = tmem + (uint32_t)(i * 128);
      const uint32_t tOi = tmem + (uint32_t)(C::kTmemO + i * D);
      const uint32_t tPi = tmem + (uint32_t)(C::kTmemP + i * C::kPStride);
      Ring<NS> ring;
      uint32_t q_par = 0, sf_par = 0, pf_par = 0, oe_par = 0;  // O-empty is first waited on for item 2
      int s_issued = 0;    // S tiles issued (the S buffer is reused every tile)
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
      auto release_unused = [&](int st) {  // a stage this sub-tile does not read
        if (lane == 0) ptx::mbar_arrive(bar(Plan::kKvEmpty + st));
        __syncwarp();
      };
      // S_i(j): kParts stages of K, each contributing its head-dim slice.
      bool pv_pending = false;  // kPAlias: a P V of this sub-tile may still be reading P (= S)
      uint32_t pvf_par = 0;
      auto do_S = [&](bool needed) -> bool {
        if (needed && s_issued > 0) {
          if (!W.wait_warp(bar(Plan::kSFree + i), sf_par)) return false;
          sf_par ^= 1;
        }
        if (C::kPAlias && needed && pv_pending) {  // S overwrites the P that P V reads
          if (!W.wait_warp(bar(Plan::kPFree + i), pvf_par)) return false;
          pvf_par ^= 1;
          pv_pending = false;
          ptx::tc_fence_after();
        }
#pragma unroll
        for (int h = 0; h < KP; ++h) {
          const int st = acquire();
          if (st < 0) return false;
          if (!needed) {
            release_unused(st);
            continue;
          }
          const uint64_t a0 = make_sdesc_sw128(sQ + h * (C::kStageCols / 64) * Plan::kChunkBytes, 16, 1024);
          const uint64_t b0 = make_sdesc_sw128(sKV + st * Plan::kStageBytes, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < C::kStageCols / 16; ++kk) {
            const uint32_t off = (uint32_t)((kk >> 2) * Plan::kChunkBytes + (kk & 3) * 32) >> 4;
            ptx::umma_ss_warp(tSi, a0 + off, b0 + off, idS, (h > 0 || kk > 0) ? 1u : 0u);
          }
          ptx::tc_commit_warp(bar(Plan::kKvEmpty + st));
        }
        if (needed) {
          ptx::tc_commit_warp(bar(Plan::kSFull + i));
          ++s_issued;
        }
        return true;
      };
      // O_i (+)= P_i(j) V(j): kParts stages of V, each producing its head-dim slice of O.
      auto do_PV = [&](bool needed, bool first, bool last) -> bool {
        if (needed) {
          if (first && !first_item) {  // the epilogue must have drained O_i
            if (!W.wait_warp(bar(Plan::kOEmpty + i), oe_par)) return false;
            oe_par ^= 1;
          }
          if (!W.wait_warp(bar(Plan::kPFull + i), pf_par)) return false;
          pf_par ^= 1;
        }
#pragma unroll
        for (int h = 0; h < KP; ++h) {
          const int st = acquire();
          if (st < 0) return false;
          if (!needed) {
            release_unused(st);
            continue;
          }
          const uint64_t b0 = make_sdesc_sw128(sKV + st * Plan::kStageBytes, Plan::kChunkBytes, 1024);
          const uint32_t dO = tOi + (uint32_t)(h * C::kStageCols);
#pragma unroll
          for (int kk = 0; kk < kBlockN / 16; ++kk) {
            const uint32_t boff = (uint32_t)(kk * 16 * 128) >> 4;
            const uint32_t acc = (!first || kk > 0) ? 1u : 0u;
            if (C::kPInTmem) {
              ptx::umma_ts_warp(dO, tPi + (uint32_t)(kk * 8), b0 + boff, idPV, acc);
            } else {
              const uint64_t a = make_sdesc_sw128(sPi + (kk >> 2) * Plan::kChunkBytes + (kk & 3) * 32, 16, 1024);
              ptx::umma_ss_warp(dO, a, b0 + boff, idPV, acc);
            }
          }
          ptx::tc_commit_warp(bar(Plan::kKvEmpty + st));
        }
        if (needed) {
          ptx::tc_commit_warp(bar(Plan::kPFree + i));
          if (last) ptx::tc_commit_warp(bar(Plan::kOFull + i));
          pv_pending = true;
        }
        return true;
      };
      ItemReader reader;
      while (ok) {
        int t;
        if (!(ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, true, t)) || t < 0) break;
        const WorkItem it = decode_item<SUB, WIN, VAR>(t, p);
        const int nb = it.nbi(i), lo = it.loi(i);  // this sub-tile reads tiles [lo, nb)
        if (nb > 0) {
          if (!(ok = W.wait_warp(bar(Plan::kQFull + i), q_par))) break;
          q_par ^= 1;
        }
        auto mine = [&](int j) { return j >= lo && j < nb; };
        if (it.nbmax > 0) ok = do_S(mine(it.jlo));  // K(jlo); an empty item (packed batch) has no tiles
        if (ok && nb > 0 && nb - 1 == it.jlo) ptx::tc_commit_warp(bar(Plan::kQEmpty + i));  // last use of Q_i
        for (int j = it.jlo; j < it.nbmax && ok; ++j) {
          if (C::kPAlias) {  // P(j) sits in S's columns: P(j) V(j) before S(j+1)
            ok = do_PV(mine(j), j == lo, j == nb - 1);  // V(j)
            if (ok && j + 1 < it.nbmax) {
              ok = do_S(mine(j + 1));  // K(j+1)
              if (ok && nb > 0 && j + 2 == nb) ptx::tc_commit_warp(bar(Plan::kQEmpty + i));  // last S_i
            }
            continue;
          }
          if (j + 1 < it.nbmax) {
            ok = do_S(mine(j + 1));  // K(j+1)
            if (ok && nb > 0 && j + 2 == nb) ptx::tc_commit_warp(bar(Plan::kQEmpty + i));  // last S_i
          }
          if (ok) ok = do_PV(mine(j), j == lo, j == nb - 1);  // V(j)
        }
        if (nb > 0) first_item = false;
      }
      // Every MMA this warp issued (and their commit arrivals) must land before the CTA
      // releases TMEM and shared memory.
      ptx::tc_commit_warp(bar(Plan::kDrain + i));
      if (lane == 0) drain_wait(bar(Plan::kDrain + i), 0, p.timeout_ns, p.status, p.host_flag);
      __syncwarp();
    } else if (warp < kWarpProd + SUB) {
      // ========================================================= producers ===
      // Producer q loads Q of sub-tile q for every item; producer 0 also fills the K/V
      // ring. Each Q buffer is refilled as soon as its own MMA warp issued the item's last
      // S, so a sub-tile starts the next item while the other is still finishing.
      if (lane == 0) {
        const int qi = warp - kWarpProd;
        const uint64_t pol_q = ptx::policy_evict_first();
        const uint64_t pol_kv = ptx::policy_evict_last();
        const uint32_t sQ = sbase + Plan::kQ + qi * Plan::kQTileBytes;
        const uint32_t sKV = sbase + Plan::kKV;
        Ring<NS> ring;
        uint32_t qe_par = 1;
        int fills = 0;  // K/V stage fills issued
        bool q_filled = false;
        bool ok = true;
        // K or V tile j of the item's sequence (rows s0 + 128 j ...).
        auto fill = [&](const CUtensorMap* map, int j, int h_idx, int b_idx, int s0) -> bool {
          for (int h = 0; h < KP; ++h) {
            const int st = ring.stage;
            const uint32_t ph = ring.phase;
            ring.next();
            if (!W.wait(bar(Plan::kKvEmpty + st), ph ^ 1)) return false;
            ptx::mbar_arrive_expect_tx(bar(Plan::kKvFull + st), (uint32_t)Plan::kStageBytes);
#pragma unroll
            for (int cc = 0; cc < C::kStageCols / 64; ++cc)
              ptx::tma_load_4d(sKV + st * Plan::kStageBytes + cc * Plan::kChunkBytes, map,
                               bar(Plan::kKvFull + st), h * C::kStageCols + cc * 64, s0 + j * kBlockN,
                               h_idx, b_idx, pol_kv);
            ++fills;
          }
          return true;
        };
        // Producer 0 schedules: it takes item indices from the shared work counter (one
        // fetch ahead, so the atomic's latency overlaps the current item) and publishes
        // them to the item ring; every other role reads the ring.
        ItemReader reader;
        int fetched = qi == 0 ? atomicAdd(p.work_counter, 1) : 0;
        int published = 0;
        while (ok) {
          int t;
          if (qi == 0) {
            const int slot = published % kItemRing;
            const uint32_t parity = ((uint32_t)(published / kItemRing) & 1u) ^ 1u;
            if (!(ok = W.wait(bar(Plan::kItemEmpty + slot), parity))) break;
            t = fetched < p.num_items ? fetched : -1;
            if (t >= 0) fetched = atomicAdd(p.work_counter, 1);
            items[slot] = t;
            ptx::mbar_arrive(bar(Plan::kItemFull + slot));  // release: publishes the slot
            ++published;
          } else if (!(ok = reader.next(W, bar(Plan::kItemFull), bar(Plan::kItemEmpty), items, false, t))) {
            break;
          }
          if (t < 0) break;
          const WorkItem it = decode_item<SUB, WIN, VAR>(t, p);
          if (it.nbi(qi) > 0) {
            if (!(ok = W.wait(bar(Plan::kQEmpty + qi), qe_par))) break;
            qe_par ^= 1;
            ptx::mbar_arrive_expect_tx(bar(Plan::kQFull + qi), (uint32_t)Plan::kQTileBytes);
            for (int cc = 0; cc < D / 64; ++cc)
              ptx::tma_load_4d(sQ + cc * Plan::kChunkBytes, &tmQ, bar(Plan::kQFull + qi), cc * 64,
                               it.s0 + it.m0 + qi * kBlockM, it.h, it.tb, pol_q);
            q_filled = true;
          }
          if (qi != 0) continue;
          const int hkv = it.h / p.kv_group;  // grouped-query attention: shared K/V head
          if (it.nbmax > 0) ok = fill(&tmK, it.jlo, hkv, it.tb, it.s0);
          for (int j = it.jlo; j < it.nbmax && ok; ++j) {
            if (C::kPAlias) {  // the MMA warps' order: V(j), then K(j+1)
              ok = fill(&tmV, j, hkv, it.tb, it.s0);
              if (ok && j + 1 < it.nbmax) ok = fill(&tmK, j + 1, hkv, it.tb, it.s0);
              continue;
            }
            if (j + 1 < it.nbmax) ok = fill(&tmK, j + 1, hkv, it.tb, it.s0);
            if (ok) ok = fill(&tmV, j, hkv, it.tb, it.s0);
          }
        }
        // Let every load this thread issued land before the CTA exits (normally they were
        // all consumed already and these waits return at once).
        const int last = fills < NS ? fills : NS;
        for (int k = 0; k < last; ++k) {
          const int f = fills - 1 - k;  // fill index
          drain_wait(bar(Plan::kKvFull + (f % NS)), (uint32_t)((f / NS) & 1), p.timeout_ns, p.status, p.host_flag);
        }
        // qe_par equals the parity of the last Q fill's phase (it flips once per fill).
        if (q_filled) drain_wait(bar(Plan::kQFull + qi), qe_par, p.timeout_ns, p.status, p.host_flag);
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
