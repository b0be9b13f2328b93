// Host side of apex_attn: argument validation, tensor-map encoding, per-device state
// and kernel dispatch behind the C ABI declared in include/apex_attn.h (forward and
// backward).
//
// The Python operator custom_attention_forward (mls-bench_fused_attention/
// fused_attention.py:155-193) did, per call: make q/k/v contiguous, default the scale,
// fold log2(e), allocate o, pick a per-head-dim config (_CONFIGS, :148-152), build TMA
// descriptors for d=128 (:165-169) and launch a grid of (ceil(N/128), B*H) programs.
// Here the caller owns every buffer; this file validates the layout, encodes 4-D TMA
// tensor maps (so strided [B,H,N,D] and [B,N,H,D] views need no copy), and launches one
// persistent CTA per SM with the per-head-dim configuration apex::Cfg<D>.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <mutex>

#include "apex_attn.h"
#include "attn_bwd_kernel.cuh"
#include "attn_fwd_kernel.cuh"
#include "attn_fwd_tile_kernel.cuh"

namespace {

using apex::AttnParams;

constexpr int kVersion = 300;  // 0.3.0

// Build-time tuning knob (overridable with -D for sweeps): exp2 pairs out of every 8 of an
// unmasked tile that use the FMA-pipe polynomial, per head dim. At d = 64 four softmax warps
// share each sub-partition and leave issue slots free beside MUFU: one pair in eight on the
// FMA pipe measured +4-5 % (C2 573-580 -> 601-604 TFLOP/s, fp16 MLS d64 651 -> 680); two
// in eight the same, three in eight slower. At d = 128, with the row-split softmax and both
// rows' max trees ahead of the rescale decisions, one in eight measures level to +2 % over
// two (C3 and the fp16 MLS d128 shape, each timed first and second in alternating
// processes); three in eight spills. d = 256 is slower with any.
#ifndef APEX_EMU64
#define APEX_EMU64 1
#endif
#ifndef APEX_EMU128
#define APEX_EMU128 1
#endif
#ifndef APEX_EMU256
#define APEX_EMU256 0
#endif
template <int D>
constexpr int kEmu = D == 64 ? APEX_EMU64 : (D == 128 ? APEX_EMU128 : APEX_EMU256);
// The same knob for the tile kernel (attn_fwd_tile_kernel), per head dim. Its softmax has
// two warps per sub-partition, so it keeps two pairs in eight at d = 128: one in eight
// measured 1.5-4 % slower on the small shapes that automatic selection gives it.
#ifndef APEX_TILE_EMU64
#define APEX_TILE_EMU64 1
#endif
#ifndef APEX_TILE_EMU128
#define APEX_TILE_EMU128 2
#endif
template <int D>
constexpr int kEmuTile = D == 64 ? APEX_TILE_EMU64 : APEX_TILE_EMU128;

// Forward kernel selection (apex_attn_set_forward_kernel): 0 = automatic, 1 = the
// two-sub-tile kernel for every call, 2 = the tile kernel wherever it applies.
std::atomic<int> g_fwd_kind{0};

constexpr int kMaxDevices = 64;
// Per-device scratch of the kernel: int[64]. Word 0 is the status word; words
// [kCounterBase, kCounterBase + kCounterSlots) are work-item counters. Each call takes the
// next slot (round robin) and zeroes it on its stream before the launch, so calls that
// run concurrently on different streams schedule with different counters.
constexpr int kStatusBytes = 256;
constexpr int kCounterBase = 32;
constexpr int kCounterSlots = 32;
static_assert((kCounterBase + kCounterSlots) * 4 <= kStatusBytes, "scratch layout");
std::atomic<unsigned> g_counter_seq{0};

struct DeviceState {
  bool ready = false;
  int* status = nullptr;
  // Mapped pinned host word that kernels set to 1 when they record a device-side error
  // (host address, and the address kernels use); null on the allocation-free path.
  int* host_flag = nullptr;
  int* host_flag_dev = nullptr;
  int num_sms = 0;
  int cc_major = 0, cc_minor = 0;
  unsigned attr_done = 0;  // bit per kernel instantiation
  unsigned attr_tile = 0;  // bit per tile-kernel instantiation
  unsigned long long attr_bwd = 0;  // bit per backward kernel instantiation
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
bool g_encode_tried = false;

unsigned long long wait_timeout_ns() {
  static const unsigned long long v = [] {
    const char* s = std::getenv("APEX_ATTN_WAIT_TIMEOUT_MS");
    long long ms = s ? std::atoll(s) : 0;
    if (ms <= 0) ms = 2000;
    return (unsigned long long)ms * 1000000ull;
  }();
  return v;
}

// Resolves cuTensorMapEncodeTiled once (caller holds g_mu).
bool resolve_encode_locked() {
  if (!g_encode_tried) {
    g_encode_tried = true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres) ==
            cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    else
      (void)cudaGetLastError();
  }
  return g_encode != nullptr;
}

// Device attributes shared by both state kinds (caller holds g_mu).
int probe_device_locked(int dev, DeviceState& s) {
  if (cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&s.cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&s.cc_minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return APEX_ATTN_ERR_NO_DEVICE;
  }
  if (s.cc_major != 10 || s.cc_minor != 0) return APEX_ATTN_ERR_UNSUPPORTED_ARCH;
  return APEX_ATTN_OK;
}

int init_device(int dev, DeviceState** out) {
  if (dev < 0 || dev >= kMaxDevices) return APEX_ATTN_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!resolve_encode_locked()) return APEX_ATTN_ERR_TENSOR_MAP;
  DeviceState& s = g_dev[dev];
  if (!s.ready) {
    int rc = probe_device_locked(dev, s);
    if (rc != APEX_ATTN_OK) return rc;
    if (cudaMalloc(&s.status, kStatusBytes) != cudaSuccess) {
      (void)cudaGetLastError();
      return APEX_ATTN_ERR_CUDA;
    }
    if (cudaMemset(s.status, 0, kStatusBytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
      (void)cudaGetLastError();
      return APEX_ATTN_ERR_CUDA;
    }
    void* hf = nullptr;
    void* hf_dev = nullptr;
    if (cudaHostAlloc(&hf, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess ||
        cudaHostGetDevicePointer(&hf_dev, hf, 0) != cudaSuccess) {
      (void)cudaGetLastError();
      return APEX_ATTN_ERR_CUDA;
    }
    *static_cast<volatile int*>(hf) = 0;
    s.host_flag = static_cast<int*>(hf);
    s.host_flag_dev = static_cast<int*>(hf_dev);
    s.ready = true;
  }
  *out = &s;
  return APEX_ATTN_OK;
}

// A kernel on this device recorded a device-side error (bounded-wait limit, teardown drain
// limit, shared-memory alignment): every later call fails with
// APEX_ATTN_ERR_DEVICE_TIMEOUT until apex_attn_device_status() reads and clears the state.
// The kernel writes the host flag when it records the error, so the first call that
// starts after that write sees it; no call synchronises for it.
int sticky_error(const DeviceState& s) {
  if (s.host_flag != nullptr && *reinterpret_cast<volatile int*>(s.host_flag) != 0)
    return APEX_ATTN_ERR_DEVICE_TIMEOUT;
  return APEX_ATTN_OK;
}

// ----------------------------------------------------------------------------
// Allocation-free state (apex_attn_fwd_noalloc).
//
// Some callers cannot call cudaMalloc: code that runs while a memory pool or an
// inference server owns the whole device budget, a plugin loaded into a host that
// forbids allocations outside its own allocator, or a real-time loop in which an
// allocation (and the device synchronisation it may imply) is not allowed. For them the
// forward kernel's scratch memory (the device status word that its bounded waits write on
// a timeout, and the scheduler's work-item counter) lives in the fixed array below
// instead of a cudaMalloc'd buffer.
//
// Every device that loads this library holds this array (256 bytes) until the process
// exits. A launch uses 8 bytes of it (the status word and one work-item counter, in the
// same layout as the cudaMalloc'd scratch of apex_attn_fwd) whatever B, H, N and D are, so
// no problem size needs more scratch than the array holds; requests outside the kernel's
// supported range are rejected with APEX_ATTN_ERR_TOO_LARGE, as by apex_attn_fwd.
//
// In host code `g_noalloc_scratch` is only a host-side stand-in for the device array,
// not a device address: a kernel given it would fault or use the wrong memory. The
// device address is obtained once per device with cudaGetSymbolAddress, with that device
// current, and passed to the kernel as a pointer.
// ----------------------------------------------------------------------------
constexpr int kNoAllocScratchBytes = 256;
constexpr int kNoAllocStatusBytes = (int)sizeof(int);
static_assert(kNoAllocScratchBytes == kStatusBytes, "the static scratch mirrors the allocated one");

static __device__ __align__(256) int g_noalloc_scratch[kNoAllocScratchBytes / sizeof(int)];

DeviceState g_noalloc_dev[kMaxDevices];  // status = device address of g_noalloc_scratch

// Per-device set-up of the allocation-free path: device attributes, the tensor-map
// encoder and the device address of the static scratch. Calls no allocating routine.
int init_device_noalloc(int dev, DeviceState** out) {
  if (dev < 0 || dev >= kMaxDevices) return APEX_ATTN_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!resolve_encode_locked()) return APEX_ATTN_ERR_TENSOR_MAP;
  DeviceState& s = g_noalloc_dev[dev];
  if (!s.ready) {
    int rc = probe_device_locked(dev, s);
    if (rc != APEX_ATTN_OK) return rc;
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) {
      (void)cudaGetLastError();
      return APEX_ATTN_ERR_CUDA;
    }
    s.status = static_cast<int*>(ptr);
    s.ready = true;
  }
  *out = &s;
  return APEX_ATTN_OK;
}

// ----------------------------------------------------------------------------

// Resolves the device that owns `ptr`; -1 when it is not device memory.
int device_of(const void* ptr) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
    (void)cudaGetLastError();
    return -1;
  }
  if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged) return -1;
  return a.device;
}

// 4-D tiled map over a logical [B, H, N, D] tensor, dims ordered (D, N, H, B), box
// (64, 128, 1, 1), 128-byte swizzle, zero fill out of bounds (rows >= N read as 0).
int encode_map(CUtensorMap* m, const void* ptr, int dtype, int B, int H, int N, int D, long long sb,
               long long sh, long long sn) {
  // Strides of size-1 dims are never used; give them a legal value.
  if (H == 1) sh = (long long)N * sn;
  if (B == 1) sb = (long long)H * sh;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)N, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)sn * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)apex::kBlockM, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(m, dtype == APEX_ATTN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        4, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? APEX_ATTN_OK : APEX_ATTN_ERR_TENSOR_MAP;
}

// Fused backward: the fp32 dQ accumulator as `planes` planes of `rows` rows x D, for TMA
// reduce-adds of 32-column x 128-row boxes (128 bytes per box row, 128-byte swizzle).
int encode_acc_map(CUtensorMap* m, float* ptr, int D, long long rows, long long planes) {
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)rows, (cuuint64_t)planes};
  cuuint64_t strides[2] = {(cuuint64_t)D * 4, (cuuint64_t)rows * D * 4};
  cuuint32_t box[3] = {32, (cuuint32_t)apex::kBlockM, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, ptr, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? APEX_ATTN_OK : APEX_ATTN_ERR_TENSOR_MAP;
}

template <int D, typename T, bool WIN, bool VAR>
int launch_one(DeviceState& ds, unsigned attr_bit, const CUtensorMap& mq, const CUtensorMap& mk,
               const CUtensorMap& mv, const AttnParams& p, int grid, cudaStream_t stream) {
  auto kern = apex::attn_fwd_sm100_kernel<D, T, kEmu<D>, WIN, VAR>;
  constexpr int smem = apex::SmemPlan<D, WIN>::kDynamicBytes;
  if (!(ds.attr_done & attr_bit)) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      (void)cudaGetLastError();
      return APEX_ATTN_ERR_LAUNCH;
    }
    ds.attr_done |= attr_bit;
  }
  kern<<<grid, apex::Cfg<D, WIN>::kThreads, smem, stream>>>(mq, mk, mv, p);
  if (cudaGetLastError() != cudaSuccess) return APEX_ATTN_ERR_LAUNCH;
  return APEX_ATTN_OK;
}

// attr_bit covers the (D, T) pair; the windowed instantiations shift it by 8, the packed
// variable-length ones by 16.
template <int D, typename T>
int launch(DeviceState& ds, unsigned attr_bit, const CUtensorMap& mq, const CUtensorMap& mk,
           const CUtensorMap& mv, const AttnParams& p, int grid, cudaStream_t stream) {
  const bool win = p.window >= 0;
  if (p.cu_seqlens != nullptr)
    return win ? launch_one<D, T, true, true>(ds, attr_bit << 24, mq, mk, mv, p, grid, stream)
               : launch_one<D, T, false, true>(ds, attr_bit << 16, mq, mk, mv, p, grid, stream);
  return win ? launch_one<D, T, true, false>(ds, attr_bit << 8, mq, mk, mv, p, grid, stream)
             : launch_one<D, T, false, false>(ds, attr_bit, mq, mk, mv, p, grid, stream);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int item_rows(int head_dim) {
  switch (head_dim) {
    case 64: return apex::Cfg<64>::kItemRows;
    case 128: return apex::Cfg<128>::kItemRows;
    default: return apex::Cfg<256>::kItemRows;
  }
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) {
      (void)cudaGetLastError();
      prev = -1;
    }
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

__global__ void wait_timeout_selftest_kernel(int* status, int* host_flag, unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    apex::ptx::mbar_init(apex::ptx::smem_u32(&bar), 1);
    abort_flag = 0;
    apex::ptx::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const apex::Waiter w{&abort_flag, status, timeout_ns, host_flag};
    (void)w.wait(apex::ptx::smem_u32(&bar), 0);  // nothing ever arrives: must time out
  }
  __syncthreads();
}

bool supported_head_dim(int head_dim) { return head_dim == 64 || head_dim == 128 || head_dim == 256; }

int schedule_and_launch(DeviceState& dst, bool noalloc, AttnParams& p, const CUtensorMap& mq,
                        const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap* mo, int head_dim,
                        int dtype, void* stream);

template <int D, typename T>
int launch_tile(DeviceState& ds, unsigned attr_bit, const CUtensorMap& mq, const CUtensorMap& mk,
                const CUtensorMap& mv, const CUtensorMap& mo, const AttnParams& p, int grid, cudaStream_t stream) {
  auto kern = apex::attn_fwd_tile_kernel<D, T, kEmuTile<D>>;
  constexpr int smem = apex::TilePlan<D>::kDynamicBytes;
  if (!(ds.attr_tile & attr_bit)) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      (void)cudaGetLastError();
      return APEX_ATTN_ERR_LAUNCH;
    }
    ds.attr_tile |= attr_bit;
  }
  kern<<<grid, apex::TileCfg<D>::kThreads, smem, stream>>>(mq, mk, mv, mo, p);
  if (cudaGetLastError() != cudaSuccess) return APEX_ATTN_ERR_LAUNCH;
  return APEX_ATTN_OK;
}

// The tile kernel covers batched launches at head dims 64 and 128 without a window; the
// two-sub-tile kernel covers the rest (d = 256, sliding windows, packed batches). Where
// both apply, automatic selection follows measurements on one B200 (bf16, causal):
//   * the tile kernel runs a 128x128 tile slower per SM (0.64x at C2, d = 64; 0.82x at C3,
//     d = 128: two softmax warps per SM sub-partition hide less latency than four);
//   * its 128-row items double the parallelism. At d = 128 and N >= 4096 that wins while
//     the problem has at most 384 256-row items (B1 H12 N8192 1111 vs 1054 TFLOP/s,
//     B1 H8 N8192 1058 vs 855, B3 H8 N4096 955 vs 917) and loses from 448 (B1 H14 N8192
//     1006 vs 1082, B2 H16 N4096 981 vs 1024, B2 H8 N8192 1076 vs 1172). At N <= 2048 the
//     shorter causal rows keep it level or ahead up to about 1024 items (B6 H16 N2048 788
//     vs 752 at 768 items, B8 H32 N1024 695 vs 662 at 1024, B8 H16 N2048 877 vs 874);
//   * at d = 64 it gains at most 8 % on small shapes and loses up to 14 %, so automatic
//     selection keeps the two-sub-tile kernel there.
bool use_tile_kernel(int head_dim, const AttnParams& p, const CUtensorMap* mo, int num_sms) {
  const int kind = g_fwd_kind.load(std::memory_order_relaxed);
  if (kind == 1 || mo == nullptr || (head_dim != 64 && head_dim != 128) || p.window >= 0 ||
      p.cu_seqlens != nullptr)
    return false;
  if (kind == 2) return true;
  const long long items = (long long)p.B * p.H * ((p.N + 2 * apex::kBlockM - 1) / (2 * apex::kBlockM));
  return head_dim == 128 && (items < 3LL * num_sms || (p.N <= 2048 && items < 8LL * num_sms));
}

// Validation, tensor maps, parameters and dispatch shared by both forward entry points.
// `noalloc` selects the allocation-free device state and clears its status word first.
int forward(bool noalloc, const void* q, const void* k, const void* v, void* o, float* lse, int batch,
            int heads, int heads_kv, int seqlen, int head_dim, int dtype, int causal, int window,
            float sm_scale, const long long* strides, void* stream) {
  // ---- argument validation (no CUDA calls) ----
  if (!q || !k || !v || !o || !strides) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (batch <= 0 || heads <= 0 || seqlen <= 0) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (heads_kv <= 0 || heads % heads_kv != 0) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (window < -1 || (window >= 0 && !causal)) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (!supported_head_dim(head_dim)) return APEX_ATTN_ERR_UNSUPPORTED_HEAD_DIM;
  if (dtype != APEX_ATTN_BF16 && dtype != APEX_ATTN_FP16) return APEX_ATTN_ERR_UNSUPPORTED_DTYPE;
  if (!std::isfinite(sm_scale) || !(sm_scale > 0.f)) return APEX_ATTN_ERR_BAD_SCALE;
  const long long BH = (long long)batch * heads;
  const long long mblocks = (seqlen + apex::kBlockM - 1) / apex::kBlockM;  // the smaller item of both kernels
  if (BH * mblocks > 0x7fffffffLL || seqlen > (1 << 30) || BH > (1LL << 30)) return APEX_ATTN_ERR_TOO_LARGE;
  for (int i = 0; i < 12; ++i)
    if (strides[i] < 0 || (strides[i] & 7) != 0 || strides[i] >= (1LL << 38)) return APEX_ATTN_ERR_BAD_LAYOUT;
  for (int t = 0; t < 4; ++t)
    if (strides[3 * t + 2] < head_dim) return APEX_ATTN_ERR_BAD_LAYOUT;  // rows must not overlap
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return APEX_ATTN_ERR_BAD_LAYOUT;
  if (lse && (reinterpret_cast<uintptr_t>(lse) & 3u)) return APEX_ATTN_ERR_BAD_LAYOUT;

  // ---- device ----
  const int dev = device_of(q);
  if (dev < 0 || device_of(k) != dev || device_of(v) != dev || device_of(o) != dev) return APEX_ATTN_ERR_NO_DEVICE;
  if (lse && device_of(lse) != dev) return APEX_ATTN_ERR_NO_DEVICE;
  DeviceGuard guard(dev);
  DeviceState* ds = nullptr;
  int rc = noalloc ? init_device_noalloc(dev, &ds) : init_device(dev, &ds);
  if (rc != APEX_ATTN_OK || (rc = sticky_error(*ds)) != APEX_ATTN_OK) return rc;

  CUtensorMap mq, mk, mv, mo;
  if ((rc = encode_map(&mq, q, dtype, batch, heads, seqlen, head_dim, strides[0], strides[1], strides[2])) ||
      (rc = encode_map(&mk, k, dtype, batch, heads_kv, seqlen, head_dim, strides[3], strides[4], strides[5])) ||
      (rc = encode_map(&mv, v, dtype, batch, heads_kv, seqlen, head_dim, strides[6], strides[7], strides[8])) ||
      (rc = encode_map(&mo, o, dtype, batch, heads, seqlen, head_dim, strides[9], strides[10], strides[11])))
    return rc;

  AttnParams p{};
  p.o = o;
  p.lse = lse;
  p.o_sb = strides[9];
  p.o_sh = strides[10];
  p.o_sn = strides[11];
  p.B = batch;
  p.H = heads;
  p.N = seqlen;
  p.kv_group = heads / heads_kv;
  // A window of seqlen or more hides nothing: the unwindowed kernels give the same result.
  p.window = window < seqlen ? window : -1;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  return schedule_and_launch(*ds, noalloc, p, mq, mk, mv, &mo, head_dim, dtype, stream);
}

// Scheduling parameters, scratch, and the launch shared by every forward entry point. The
// caller filled the output, shape, mask and scale fields of p.
int schedule_and_launch(DeviceState& dst, bool noalloc, AttnParams& p, const CUtensorMap& mq,
                        const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap* mo, int head_dim,
                        int dtype, void* stream) {
  DeviceState* ds = &dst;
  const long long BH = (long long)p.B * p.H;
  const bool tile = use_tile_kernel(head_dim, p, mo, ds->num_sms);
  const int rows_per_item = tile ? apex::kBlockM : item_rows(head_dim);
  const long long mblocks = (p.N + rows_per_item - 1) / rows_per_item;
  p.status = ds->status;
  p.host_flag = ds->host_flag_dev;
  p.num_mblocks = (int)mblocks;
  p.num_kblocks = (p.N + apex::kBlockN - 1) / apex::kBlockN;
  p.num_items = (int)(BH * mblocks);
  // L2 scheduling groups: keep the K/V of the heads that concurrently running CTAs stream
  // within ~48 MB of L2 (query heads that share a K/V head count once); split the heads
  // into groups whose sizes differ by at most one.
  const double kv_bytes_per_head = 2.0 * p.N * head_dim * 2.0 / p.kv_group;
  long long g = (long long)(48.0 * 1024 * 1024 / kv_bytes_per_head);
  g = std::max(1LL, std::min(g, BH));
  long long ngroups = (BH + g - 1) / g;
  // Load balance across the groups: items run longest first inside a group, but the groups
  // run one after another, so the last group's longest item starts when about
  // (1 - 1/ngroups) of the work is done and must fit in the work left. Allow at most
  // (work per SM) / (1.25 x longest item) groups; item work counts the K/V tiles of its
  // busiest sub-tile. Shapes with many items per SM are not limited (the bound is only
  // evaluated up to 4096 query blocks). Measured against the L2 bound alone: the MLS
  // shapes d=128 (32 heads, N=8192) 3 -> 2 groups +2-3 % and d=256 (8 heads, N=16384)
  // 3 -> 2 groups +8-9 %; C3 keeps its 11 groups (a factor of 1.5 would give 9, -0.5 %).
  if (ngroups > 1 && mblocks <= 4096) {
    const int sub_rows = apex::kBlockM;
    const int ksub = rows_per_item / sub_rows;
    double sum_tiles = 0.0;
    long long max_tiles = 1;
    for (long long mb = 0; mb < mblocks; ++mb) {
      long long tiles = 0;
      for (int i = 0; i < ksub; ++i) {
        const long long r0 = mb * rows_per_item + (long long)i * sub_rows;
        if (r0 >= p.N) break;
        const long long nb = p.causal ? std::min<long long>(p.num_kblocks, r0 / apex::kBlockN + 1) : p.num_kblocks;
        const long long lo = p.window >= 0 ? std::max<long long>(0, r0 - p.window) / apex::kBlockN : 0;
        tiles = std::max(tiles, nb - lo);
      }
      sum_tiles += (double)tiles;
      max_tiles = std::max(max_tiles, tiles);
    }
    const double work_per_sm = (double)BH * sum_tiles / std::max(1, ds->num_sms);
    const long long balance = std::max(1LL, (long long)(work_per_sm / (1.25 * (double)max_tiles)));
    ngroups = std::min(ngroups, balance);
  }
  p.group_q = (int)(BH / ngroups);
  p.group_big = (int)(BH % ngroups);
  p.work_counter = ds->status + kCounterBase + (int)(g_counter_seq.fetch_add(1) % kCounterSlots);
  p.timeout_ns = wait_timeout_ns();
  const int grid = std::min(p.num_items, ds->num_sms);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  if (noalloc) {
    // The static scratch keeps the previous call's contents: the status word must start
    // at zero.
    if (cudaMemsetAsync(ds->status, 0, kNoAllocStatusBytes, s) != cudaSuccess) {
      (void)cudaGetLastError();
      return APEX_ATTN_ERR_CUDA;
    }
  }
  // The work counter must start at zero (ordered before the kernel on the same stream).
  if (cudaMemsetAsync(p.work_counter, 0, sizeof(int), s) != cudaSuccess) {
    (void)cudaGetLastError();
    return APEX_ATTN_ERR_CUDA;
  }
  const bool bf16 = dtype == APEX_ATTN_BF16;
  if (tile) {
    if (head_dim == 64)
      return bf16 ? launch_tile<64, __nv_bfloat16>(*ds, 1u, mq, mk, mv, *mo, p, grid, s)
                  : launch_tile<64, __half>(*ds, 2u, mq, mk, mv, *mo, p, grid, s);
    return bf16 ? launch_tile<128, __nv_bfloat16>(*ds, 4u, mq, mk, mv, *mo, p, grid, s)
                : launch_tile<128, __half>(*ds, 8u, mq, mk, mv, *mo, p, grid, s);
  }
  switch (head_dim) {
    case 64:
      return bf16 ? launch<64, __nv_bfloat16>(*ds, 1u, mq, mk, mv, p, grid, s)
                  : launch<64, __half>(*ds, 2u, mq, mk, mv, p, grid, s);
    case 128:
      return bf16 ? launch<128, __nv_bfloat16>(*ds, 4u, mq, mk, mv, p, grid, s)
                  : launch<128, __half>(*ds, 8u, mq, mk, mv, p, grid, s);
    default:
      return bf16 ? launch<256, __nv_bfloat16>(*ds, 16u, mq, mk, mv, p, grid, s)
                  : launch<256, __half>(*ds, 32u, mq, mk, mv, p, grid, s);
  }
}

// Packed variable-length forward (apex_attn_fwd_varlen).
int forward_varlen(const apex_attn_varlen_args* a, void* stream) {
  // ---- argument validation (no CUDA calls) ----
  if (!a || !a->q || !a->k || !a->v || !a->o || !a->cu_seqlens) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (a->batch <= 0 || a->heads_q <= 0 || a->total <= 0 || a->max_seqlen <= 0)
    return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (a->heads_kv <= 0 || a->heads_q % a->heads_kv != 0) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (a->window_left < -1 || (a->window_left >= 0 && !a->causal)) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (!supported_head_dim(a->head_dim)) return APEX_ATTN_ERR_UNSUPPORTED_HEAD_DIM;
  if (a->dtype != APEX_ATTN_BF16 && a->dtype != APEX_ATTN_FP16) return APEX_ATTN_ERR_UNSUPPORTED_DTYPE;
  if (!std::isfinite(a->sm_scale) || !(a->sm_scale > 0.f)) return APEX_ATTN_ERR_BAD_SCALE;
  const long long mblocks = (a->max_seqlen + item_rows(a->head_dim) - 1) / item_rows(a->head_dim);
  if ((long long)a->batch * a->heads_q * mblocks > 0x7fffffffLL || a->total > (1 << 30) ||
      a->max_seqlen > (1 << 30) || a->batch > (1 << 30))
    return APEX_ATTN_ERR_TOO_LARGE;
  for (int i = 0; i < 8; ++i)
    if (a->strides[i] < 0 || (a->strides[i] & 7) != 0 || a->strides[i] >= (1LL << 38)) return APEX_ATTN_ERR_BAD_LAYOUT;
  for (int t = 0; t < 4; ++t)  // (token, head) per tensor: rows of one token must not overlap
    if (a->strides[2 * t + 1] < a->head_dim) return APEX_ATTN_ERR_BAD_LAYOUT;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o)) return APEX_ATTN_ERR_BAD_LAYOUT;
  if ((a->lse && (reinterpret_cast<uintptr_t>(a->lse) & 3u)) || (reinterpret_cast<uintptr_t>(a->cu_seqlens) & 3u))
    return APEX_ATTN_ERR_BAD_LAYOUT;

  // ---- device ----
  const int dev = device_of(a->q);
  if (dev < 0 || device_of(a->k) != dev || device_of(a->v) != dev || device_of(a->o) != dev ||
      device_of(a->cu_seqlens) != dev)
    return APEX_ATTN_ERR_NO_DEVICE;
  if (a->lse && device_of(a->lse) != dev) return APEX_ATTN_ERR_NO_DEVICE;
  DeviceGuard guard(dev);
  DeviceState* ds = nullptr;
  int rc = init_device(dev, &ds);
  if (rc != APEX_ATTN_OK || (rc = sticky_error(*ds)) != APEX_ATTN_OK) return rc;

  // One 4-D map per tensor over the packed rows: dims (D, total, H, 1).
  const long long* st = a->strides;
  CUtensorMap mq, mk, mv;
  if ((rc = encode_map(&mq, a->q, a->dtype, 1, a->heads_q, a->total, a->head_dim, 0, st[1], st[0])) ||
      (rc = encode_map(&mk, a->k, a->dtype, 1, a->heads_kv, a->total, a->head_dim, 0, st[3], st[2])) ||
      (rc = encode_map(&mv, a->v, a->dtype, 1, a->heads_kv, a->total, a->head_dim, 0, st[5], st[4])))
    return rc;
  AttnParams p{};
  p.o = a->o;
  p.lse = a->lse;
  p.o_sb = 0;
  p.o_sh = st[7];
  p.o_sn = st[6];
  p.B = a->batch;
  p.H = a->heads_q;
  p.N = a->max_seqlen;
  p.kv_group = a->heads_q / a->heads_kv;
  p.window = a->window_left < a->max_seqlen ? a->window_left : -1;  // wider hides nothing
  p.causal = a->causal ? 1 : 0;
  p.scale_log2 = a->sm_scale * 1.4426950408889634f;
  p.cu_seqlens = a->cu_seqlens;
  p.total = a->total;
  return schedule_and_launch(*ds, false, p, mq, mk, mv, nullptr, a->head_dim, a->dtype, stream);
}

// ------------------------------------------------------------------ backward --
constexpr int kBwdBlock = apex::kBlockM;

long long bwd_padded_rows(int seqlen) { return ((long long)seqlen + kBwdBlock - 1) / kBwdBlock * kBwdBlock; }

// Workspace: -lse2 then -delta, each fp32 [batch * heads_q][Npad].
size_t bwd_workspace_bytes(int batch, int heads_q, int seqlen) {
  if (batch <= 0 || heads_q <= 0 || seqlen <= 0) return 0;
  return (size_t)2 * (size_t)batch * (size_t)heads_q * (size_t)bwd_padded_rows(seqlen) * sizeof(float);
}

// Fused mode: the statistics, then (256-byte aligned) the fp32 dQ accumulator of
// batch * heads_q * seqlen rows of head_dim (for a packed batch, seqlen = the longest
// sequence, so the total token count fits).
size_t bwd_dq_acc_offset(int batch, int heads_q, int seqlen) {
  return (bwd_workspace_bytes(batch, heads_q, seqlen) + 255) / 256 * 256;
}

size_t bwd_workspace_bytes_mode(int batch, int heads_q, int seqlen, int head_dim, int mode) {
  if (batch <= 0 || heads_q <= 0 || seqlen <= 0) return 0;
  if (mode != APEX_ATTN_BWD_FUSED) return bwd_workspace_bytes(batch, heads_q, seqlen);
  if (head_dim <= 0) return 0;
  return bwd_dq_acc_offset(batch, heads_q, seqlen) +
         (size_t)batch * (size_t)heads_q * (size_t)seqlen * (size_t)head_dim * sizeof(float);
}

// The backward's inputs in one shape for the batched and the packed entry points: strides
// are (batch, head, row) element strides of q, k, v, o, dout, dq, dk, dv (batch stride 0
// for a packed batch, whose rows are tokens).
struct BwdCall {
  const void *o, *dout;
  const float* lse;
  void *dq, *dk, *dv;
  int batch, heads_q, heads_kv, seqlen, causal, window_left;  // seqlen: the longest sequence
  float sm_scale;
  long long st[24];
  const int* cu_seqlens;  // null: batched
  int total;
  float* dq_acc;  // fused mode: the zeroed fp32 dQ accumulator; null: two passes
};

template <int D, typename T, bool KV, bool WIN, bool VAR, bool DQ>
int launch_bwd_one(DeviceState& ds, const CUtensorMap& x1, const CUtensorMap& x2, const CUtensorMap& y1,
                   const CUtensorMap& y2, const CUtensorMap& dqm, const apex::BwdParams& p, int grid,
                   cudaStream_t stream) {
  auto kern = apex::attn_bwd_sm100_kernel<D, T, KV, WIN, VAR, DQ>;
  constexpr int smem = apex::BwdSmem<D, DQ>::kDynamicBytes;
  // One bit per instantiation: VAR, d = 128, fp16 and DQ select a group of 4 (KV, WIN).
  constexpr unsigned long long bit = 1ull << (((VAR ? 8 : 0) + (D == 128 ? 4 : 0) + (std::is_same<T, __half>::value ? 2 : 0) +
                                   (DQ ? 1 : 0)) * 4 + (KV ? 2 : 0) + (WIN ? 1 : 0));
  if (!(ds.attr_bwd & bit)) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      (void)cudaGetLastError();
      return APEX_ATTN_ERR_LAUNCH;
    }
    ds.attr_bwd |= bit;
  }
  kern<<<grid, apex::BwdCfg<D, DQ>::kThreads, smem, stream>>>(x1, x2, y1, y2, dqm, p);
  if (cudaGetLastError() != cudaSuccess) return APEX_ATTN_ERR_LAUNCH;
  return APEX_ATTN_OK;
}

// One pass (dK/dV, fused dK/dV/dQ, or dQ), windowed or not. `dqm` is read by the fused
// pass only (the others get any valid map).
template <int D, typename T, bool KV, bool VAR, bool DQ = false>
int launch_bwd_pass(DeviceState& ds, bool win, const CUtensorMap& x1, const CUtensorMap& x2,
                    const CUtensorMap& y1, const CUtensorMap& y2, const CUtensorMap& dqm,
                    const apex::BwdParams& p, int grid, cudaStream_t s) {
  return win ? launch_bwd_one<D, T, KV, true, VAR, DQ>(ds, x1, x2, y1, y2, dqm, p, grid, s)
             : launch_bwd_one<D, T, KV, false, VAR, DQ>(ds, x1, x2, y1, y2, dqm, p, grid, s);
}

// Prep pass, then the dK/dV pass (K, V stationary) and the dQ pass (Q, dO stationary).
template <int D, typename T>
int launch_bwd(DeviceState& ds, const BwdCall& a, const CUtensorMap& mq, const CUtensorMap& mk,
               const CUtensorMap& mv, const CUtensorMap& mdo, float* lse2, float* delta, cudaStream_t s) {
  const long long* st = a.st;
  const bool var = a.cu_seqlens != nullptr;
  const int npad = (int)bwd_padded_rows(a.seqlen);
  const long long rows = (long long)a.batch * a.heads_q * npad;
  const long long threads = rows * (D / 8);
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  if (var)
    apex::attn_bwd_prep_kernel<T, D, true><<<blocks, 256, 0, s>>>(
        static_cast<const T*>(a.o), static_cast<const T*>(a.dout), a.lse, lse2, delta, st[9], st[10], st[11],
        st[12], st[13], st[14], a.heads_q, a.seqlen, npad, rows, a.cu_seqlens, a.total);
  else
    apex::attn_bwd_prep_kernel<T, D, false><<<blocks, 256, 0, s>>>(
        static_cast<const T*>(a.o), static_cast<const T*>(a.dout), a.lse, lse2, delta, st[9], st[10], st[11],
        st[12], st[13], st[14], a.heads_q, a.seqlen, npad, rows, nullptr, 0);
  if (cudaGetLastError() != cudaSuccess) return APEX_ATTN_ERR_LAUNCH;

  apex::BwdParams p{};
  p.nlse2 = lse2;
  p.ndelta = delta;
  p.status = ds.status;
  p.host_flag = ds.host_flag_dev;
  p.B = a.batch;
  p.H = a.heads_q;
  p.Hkv = a.heads_kv;
  p.N = a.seqlen;
  p.Npad = npad;
  p.nblk = npad / kBwdBlock;
  p.kv_group = a.heads_q / a.heads_kv;
  p.scale_log2 = a.sm_scale * 1.4426950408889634f;
  p.out1_scale = a.sm_scale;
  p.causal = a.causal ? 1 : 0;
  // A window of seqlen or more hides nothing: run the plain causal kernels (this also keeps
  // the kernels' window arithmetic far from int overflow).
  p.window = a.window_left < a.seqlen ? a.window_left : -1;
  p.cu_seqlens = a.cu_seqlens;
  p.total = a.total;
  p.timeout_ns = wait_timeout_ns();
  // L2 groups as in the forward: the streamed tiles of the heads that concurrently running
  // CTAs walk should stay within ~48 MB of L2.
  auto set_groups = [&](apex::BwdParams& q, long long heads, double stream_bytes_per_head) {
    long long g = (long long)(48.0 * 1024 * 1024 / stream_bytes_per_head);
    g = std::max(1LL, std::min(g, heads));
    const long long ngroups = (heads + g - 1) / g;
    q.group_q = (int)(heads / ngroups);
    q.group_big = (int)(heads % ngroups);
    q.num_items = (int)(heads * q.nblk);
  };
  const bool win = p.window >= 0;
  int rc;
  // dK, dV: items over (batch, K/V head, key block); Q and dO of the group stream.
  apex::BwdParams pk = p;
  pk.out1 = a.dk;
  pk.out2 = a.dv;
  pk.o1_sb = st[18]; pk.o1_sh = st[19]; pk.o1_sn = st[20];
  pk.o2_sb = st[21]; pk.o2_sh = st[22]; pk.o2_sn = st[23];
  set_groups(pk, (long long)a.batch * a.heads_kv, 2.0 * npad * D * 2.0 * pk.kv_group);
  pk.work_counter = ds.status + kCounterBase + (int)(g_counter_seq.fetch_add(1) % kCounterSlots);
  if (cudaMemsetAsync(pk.work_counter, 0, sizeof(int), s) != cudaSuccess) {
    (void)cudaGetLastError();
    return APEX_ATTN_ERR_CUDA;
  }
  const int grid_kv = std::min(pk.num_items, ds.num_sms);
  if (a.dq_acc != nullptr) {
    // Fused: one pass adds every step's dQ tile into the zeroed fp32 accumulator, then a
    // cast writes dq = scale * acc.
    const long long acc_rows = var ? (long long)a.heads_q * a.total : (long long)a.batch * a.heads_q * a.seqlen;
    if (cudaMemsetAsync(a.dq_acc, 0, (size_t)acc_rows * D * sizeof(float), s) != cudaSuccess) {
      (void)cudaGetLastError();
      return APEX_ATTN_ERR_CUDA;
    }
    pk.dq_acc = a.dq_acc;
    CUtensorMap macc;
    rc = var ? encode_acc_map(&macc, a.dq_acc, D, a.total, a.heads_q)
             : encode_acc_map(&macc, a.dq_acc, D, a.seqlen, (long long)a.batch * a.heads_q);
    if (rc != APEX_ATTN_OK) return rc;
    rc = var ? launch_bwd_pass<D, T, true, true, true>(ds, win, mk, mv, mq, mdo, macc, pk, grid_kv, s)
             : launch_bwd_pass<D, T, true, false, true>(ds, win, mk, mv, mq, mdo, macc, pk, grid_kv, s);
    if (rc != APEX_ATTN_OK) return rc;
    if (var)
      apex::attn_bwd_dq_cast_kernel<T, D, true><<<blocks, 256, 0, s>>>(
          a.dq_acc, static_cast<T*>(a.dq), 0, st[16], st[17], a.heads_q, a.seqlen, npad, rows, a.cu_seqlens,
          a.total, a.sm_scale);
    else
      apex::attn_bwd_dq_cast_kernel<T, D, false><<<blocks, 256, 0, s>>>(
          a.dq_acc, static_cast<T*>(a.dq), st[15], st[16], st[17], a.heads_q, a.seqlen, npad, rows, nullptr, 0,
          a.sm_scale);
    return cudaGetLastError() == cudaSuccess ? APEX_ATTN_OK : APEX_ATTN_ERR_LAUNCH;
  }
  rc = var ? launch_bwd_pass<D, T, true, true>(ds, win, mk, mv, mq, mdo, mk, pk, grid_kv, s)
           : launch_bwd_pass<D, T, true, false>(ds, win, mk, mv, mq, mdo, mk, pk, grid_kv, s);
  if (rc != APEX_ATTN_OK) return rc;
  // dQ: items over (batch, query head, query block); K and V stream.
  apex::BwdParams pq = p;
  pq.out1 = a.dq;
  pq.o1_sb = st[15]; pq.o1_sh = st[16]; pq.o1_sn = st[17];
  set_groups(pq, (long long)a.batch * a.heads_q, 2.0 * npad * D * 2.0 / pq.kv_group);
  pq.work_counter = ds.status + kCounterBase + (int)(g_counter_seq.fetch_add(1) % kCounterSlots);
  if (cudaMemsetAsync(pq.work_counter, 0, sizeof(int), s) != cudaSuccess) {
    (void)cudaGetLastError();
    return APEX_ATTN_ERR_CUDA;
  }
  const int grid_q = std::min(pq.num_items, ds.num_sms);
  return var ? launch_bwd_pass<D, T, false, true>(ds, win, mq, mdo, mk, mv, mq, pq, grid_q, s)
             : launch_bwd_pass<D, T, false, false>(ds, win, mq, mdo, mk, mv, mq, pq, grid_q, s);
}

int dispatch_bwd(DeviceState& ds, const BwdCall& call, int head_dim, int dtype, const CUtensorMap& mq,
                 const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mdo, void* workspace,
                 long long npad, void* stream);

int backward(const apex_attn_bwd_args* a, int mode, void* workspace, size_t workspace_bytes, void* stream) {
  // ---- argument validation (no CUDA calls) ----
  if (!a) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (mode != APEX_ATTN_BWD_DETERMINISTIC && mode != APEX_ATTN_BWD_FUSED) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (!a->q || !a->k || !a->v || !a->o || !a->dout || !a->lse || !a->dq || !a->dk || !a->dv || !workspace)
    return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (a->batch <= 0 || a->heads_q <= 0 || a->seqlen <= 0) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (a->heads_kv <= 0 || a->heads_q % a->heads_kv != 0) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (a->window_left < -1 || (a->window_left >= 0 && !a->causal)) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (a->head_dim != 64 && a->head_dim != 128) return APEX_ATTN_ERR_UNSUPPORTED_HEAD_DIM;
  if (a->dtype != APEX_ATTN_BF16 && a->dtype != APEX_ATTN_FP16) return APEX_ATTN_ERR_UNSUPPORTED_DTYPE;
  if (!std::isfinite(a->sm_scale) || !(a->sm_scale > 0.f)) return APEX_ATTN_ERR_BAD_SCALE;
  const long long npad = bwd_padded_rows(a->seqlen);
  const long long items = (long long)a->batch * a->heads_q * (npad / kBwdBlock);
  if (items > 0x7fffffffLL || a->seqlen > (1 << 30) || (long long)a->batch * a->heads_q * npad > (1LL << 40))
    return APEX_ATTN_ERR_TOO_LARGE;
  for (int i = 0; i < 24; ++i)
    if (a->strides[i] < 0 || (a->strides[i] & 7) != 0 || a->strides[i] >= (1LL << 38)) return APEX_ATTN_ERR_BAD_LAYOUT;
  for (int t = 0; t < 8; ++t)
    if (a->strides[3 * t + 2] < a->head_dim) return APEX_ATTN_ERR_BAD_LAYOUT;
  const void* ptrs[8] = {a->q, a->k, a->v, a->o, a->dout, a->dq, a->dk, a->dv};
  for (const void* ptr : ptrs)
    if (!aligned16(ptr)) return APEX_ATTN_ERR_BAD_LAYOUT;
  if ((reinterpret_cast<uintptr_t>(a->lse) & 3u) || !aligned16(workspace)) return APEX_ATTN_ERR_BAD_LAYOUT;
  if (workspace_bytes < bwd_workspace_bytes_mode(a->batch, a->heads_q, a->seqlen, a->head_dim, mode))
    return APEX_ATTN_ERR_INVALID_ARGUMENT;

  // ---- device ----
  const int dev = device_of(a->q);
  if (dev < 0) return APEX_ATTN_ERR_NO_DEVICE;
  for (const void* ptr : ptrs)
    if (device_of(ptr) != dev) return APEX_ATTN_ERR_NO_DEVICE;
  if (device_of(a->lse) != dev || device_of(workspace) != dev) return APEX_ATTN_ERR_NO_DEVICE;
  DeviceGuard guard(dev);
  DeviceState* ds = nullptr;
  int rc = init_device(dev, &ds);
  if (rc != APEX_ATTN_OK || (rc = sticky_error(*ds)) != APEX_ATTN_OK) return rc;

  const long long* st = a->strides;
  const int B = a->batch, H = a->heads_q, HKV = a->heads_kv, N = a->seqlen, D = a->head_dim;
  CUtensorMap mq, mk, mv, mdo;
  if ((rc = encode_map(&mq, a->q, a->dtype, B, H, N, D, st[0], st[1], st[2])) ||
      (rc = encode_map(&mk, a->k, a->dtype, B, HKV, N, D, st[3], st[4], st[5])) ||
      (rc = encode_map(&mv, a->v, a->dtype, B, HKV, N, D, st[6], st[7], st[8])) ||
      (rc = encode_map(&mdo, a->dout, a->dtype, B, H, N, D, st[12], st[13], st[14])))
    return rc;
  BwdCall call{a->o, a->dout, a->lse, a->dq, a->dk, a->dv, B, H, HKV, N, a->causal, a->window_left,
               a->sm_scale, {}, nullptr, 0, nullptr};
  for (int i = 0; i < 24; ++i) call.st[i] = st[i];
  if (mode == APEX_ATTN_BWD_FUSED)
    call.dq_acc = reinterpret_cast<float*>(static_cast<char*>(workspace) + bwd_dq_acc_offset(B, H, N));
  return dispatch_bwd(*ds, call, a->head_dim, a->dtype, mq, mk, mv, mdo, workspace, npad, stream);
}

int dispatch_bwd(DeviceState& ds, const BwdCall& call, int head_dim, int dtype, const CUtensorMap& mq,
                 const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mdo, void* workspace,
                 long long npad, void* stream) {
  float* lse2 = static_cast<float*>(workspace);
  float* delta = lse2 + (size_t)call.batch * call.heads_q * npad;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool bf16 = dtype == APEX_ATTN_BF16;
  if (head_dim == 64)
    return bf16 ? launch_bwd<64, __nv_bfloat16>(ds, call, mq, mk, mv, mdo, lse2, delta, s)
                : launch_bwd<64, __half>(ds, call, mq, mk, mv, mdo, lse2, delta, s);
  return bf16 ? launch_bwd<128, __nv_bfloat16>(ds, call, mq, mk, mv, mdo, lse2, delta, s)
              : launch_bwd<128, __half>(ds, call, mq, mk, mv, mdo, lse2, delta, s);
}

// Packed variable-length backward (apex_attn_bwd_varlen).
int backward_varlen(const apex_attn_bwd_varlen_args* a, int mode, void* workspace, size_t workspace_bytes,
                    void* stream) {
  // ---- argument validation (no CUDA calls) ----
  if (!a) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (mode != APEX_ATTN_BWD_DETERMINISTIC && mode != APEX_ATTN_BWD_FUSED) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (!a->q || !a->k || !a->v || !a->o || !a->dout || !a->lse || !a->dq || !a->dk || !a->dv ||
      !a->cu_seqlens || !workspace)
    return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (a->batch <= 0 || a->heads_q <= 0 || a->total <= 0 || a->max_seqlen <= 0) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (a->heads_kv <= 0 || a->heads_q % a->heads_kv != 0) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (a->window_left < -1 || (a->window_left >= 0 && !a->causal)) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (a->head_dim != 64 && a->head_dim != 128) return APEX_ATTN_ERR_UNSUPPORTED_HEAD_DIM;
  if (a->dtype != APEX_ATTN_BF16 && a->dtype != APEX_ATTN_FP16) return APEX_ATTN_ERR_UNSUPPORTED_DTYPE;
  if (!std::isfinite(a->sm_scale) || !(a->sm_scale > 0.f)) return APEX_ATTN_ERR_BAD_SCALE;
  const long long npad = bwd_padded_rows(a->max_seqlen);
  if ((long long)a->batch * a->heads_q * (npad / kBwdBlock) > 0x7fffffffLL || a->total > (1 << 30) ||
      a->max_seqlen > (1 << 30) || (long long)a->batch * a->heads_q * npad > (1LL << 40))
    return APEX_ATTN_ERR_TOO_LARGE;
  for (int i = 0; i < 16; ++i)
    if (a->strides[i] < 0 || (a->strides[i] & 7) != 0 || a->strides[i] >= (1LL << 38)) return APEX_ATTN_ERR_BAD_LAYOUT;
  for (int t = 0; t < 8; ++t)
    if (a->strides[2 * t + 1] < a->head_dim) return APEX_ATTN_ERR_BAD_LAYOUT;
  const void* ptrs[8] = {a->q, a->k, a->v, a->o, a->dout, a->dq, a->dk, a->dv};
  for (const void* ptr : ptrs)
    if (!aligned16(ptr)) return APEX_ATTN_ERR_BAD_LAYOUT;
  if ((reinterpret_cast<uintptr_t>(a->lse) & 3u) || (reinterpret_cast<uintptr_t>(a->cu_seqlens) & 3u) ||
      !aligned16(workspace))
    return APEX_ATTN_ERR_BAD_LAYOUT;
  // The fused mode's accumulator holds heads_q x total rows; total <= batch x max_seqlen
  // for valid offsets, and the size asked for covers batch x max_seqlen.
  if (mode == APEX_ATTN_BWD_FUSED && (long long)a->total > (long long)a->batch * a->max_seqlen)
    return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < bwd_workspace_bytes_mode(a->batch, a->heads_q, a->max_seqlen, a->head_dim, mode))
    return APEX_ATTN_ERR_INVALID_ARGUMENT;

  // ---- device ----
  const int dev = device_of(a->q);
  if (dev < 0) return APEX_ATTN_ERR_NO_DEVICE;
  for (const void* ptr : ptrs)
    if (device_of(ptr) != dev) return APEX_ATTN_ERR_NO_DEVICE;
  if (device_of(a->lse) != dev || device_of(a->cu_seqlens) != dev || device_of(workspace) != dev)
    return APEX_ATTN_ERR_NO_DEVICE;
  DeviceGuard guard(dev);
  DeviceState* ds = nullptr;
  int rc = init_device(dev, &ds);
  if (rc != APEX_ATTN_OK || (rc = sticky_error(*ds)) != APEX_ATTN_OK) return rc;

  // Tensor maps over the packed rows: dims (D, total, H, 1); strides are (token, head).
  const long long* st = a->strides;
  const int T = a->total, D = a->head_dim;
  CUtensorMap mq, mk, mv, mdo;
  if ((rc = encode_map(&mq, a->q, a->dtype, 1, a->heads_q, T, D, 0, st[1], st[0])) ||
      (rc = encode_map(&mk, a->k, a->dtype, 1, a->heads_kv, T, D, 0, st[3], st[2])) ||
      (rc = encode_map(&mv, a->v, a->dtype, 1, a->heads_kv, T, D, 0, st[5], st[4])) ||
      (rc = encode_map(&mdo, a->dout, a->dtype, 1, a->heads_q, T, D, 0, st[9], st[8])))
    return rc;
  BwdCall call{a->o, a->dout, a->lse, a->dq, a->dk, a->dv, a->batch, a->heads_q, a->heads_kv,
               a->max_seqlen, a->causal, a->window_left, a->sm_scale, {}, a->cu_seqlens, a->total, nullptr};
  if (mode == APEX_ATTN_BWD_FUSED)
    call.dq_acc = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                           bwd_dq_acc_offset(a->batch, a->heads_q, a->max_seqlen));
  for (int t = 0; t < 8; ++t) {  // (batch, head, row) per tensor; no batch stride when packed
    call.st[3 * t] = 0;
    call.st[3 * t + 1] = st[2 * t + 1];
    call.st[3 * t + 2] = st[2 * t];
  }
  return dispatch_bwd(*ds, call, a->head_dim, a->dtype, mq, mk, mv, mdo, workspace, npad, stream);
}

}  // namespace

extern "C" {

size_t apex_attn_bwd_workspace_bytes(int batch, int heads_q, int seqlen) {
  return bwd_workspace_bytes(batch, heads_q, seqlen);
}

size_t apex_attn_bwd_workspace_bytes_mode(int batch, int heads_q, int seqlen, int head_dim, int mode) {
  return bwd_workspace_bytes_mode(batch, heads_q, seqlen, head_dim, mode);
}

int apex_attn_bwd(const apex_attn_bwd_args* args, void* workspace, size_t workspace_bytes, void* stream) {
  return backward(args, APEX_ATTN_BWD_DETERMINISTIC, workspace, workspace_bytes, stream);
}

int apex_attn_bwd_mode(const apex_attn_bwd_args* args, int mode, void* workspace, size_t workspace_bytes,
                       void* stream) {
  return backward(args, mode, workspace, workspace_bytes, stream);
}

int apex_attn_bwd_varlen(const apex_attn_bwd_varlen_args* args, void* workspace, size_t workspace_bytes,
                         void* stream) {
  return backward_varlen(args, APEX_ATTN_BWD_DETERMINISTIC, workspace, workspace_bytes, stream);
}

int apex_attn_bwd_varlen_mode(const apex_attn_bwd_varlen_args* args, int mode, void* workspace,
                              size_t workspace_bytes, void* stream) {
  return backward_varlen(args, mode, workspace, workspace_bytes, stream);
}

int apex_attn_version(void) { return kVersion; }

int apex_attn_supports_head_dim(int head_dim) { return supported_head_dim(head_dim) ? 1 : 0; }

const char* apex_attn_strerror(int status) {
  switch (status) {
    case APEX_ATTN_OK: return "success";
    case APEX_ATTN_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer or non-positive size)";
    case APEX_ATTN_ERR_UNSUPPORTED_HEAD_DIM: return "unsupported head dim (supported: 64, 128, 256)";
    case APEX_ATTN_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype (supported: bf16, fp16)";
    case APEX_ATTN_ERR_BAD_LAYOUT: return "layout not supported: head-dim stride must be 1, other strides multiples of 8 elements, pointers 16-byte aligned";
    case APEX_ATTN_ERR_BAD_SCALE: return "sm_scale must be finite and > 0";
    case APEX_ATTN_ERR_NO_DEVICE: return "tensors are not CUDA device memory on one device";
    case APEX_ATTN_ERR_UNSUPPORTED_ARCH: return "device is not sm_100 (B200)";
    case APEX_ATTN_ERR_TENSOR_MAP: return "TMA tensor map encoding failed";
    case APEX_ATTN_ERR_LAUNCH: return "kernel launch failed";
    case APEX_ATTN_ERR_DEVICE_TIMEOUT: return "a kernel on this device reported a device-side error (bounded-wait timeout, teardown drain limit or shared-memory alignment); its outputs are incomplete. apex_attn_device_status() reads and clears the state";
    case APEX_ATTN_ERR_TOO_LARGE: return "sizes exceed the supported range";
    case APEX_ATTN_ERR_CUDA: return "CUDA runtime error";
    default: return "unknown status";
  }
}

int apex_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int batch,
                  int heads, int seqlen, int head_dim, int dtype, int causal, float sm_scale,
                  const long long* strides, void* stream) {
  return forward(false, q, k, v, o, lse, batch, heads, heads, seqlen, head_dim, dtype, causal, -1,
                 sm_scale, strides, stream);
}

int apex_attn_fwd_ex(const apex_attn_fwd_args* a, void* stream) {
  if (!a) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  return forward(false, a->q, a->k, a->v, a->o, a->lse, a->batch, a->heads_q, a->heads_kv, a->seqlen,
                 a->head_dim, a->dtype, a->causal, a->window_left, a->sm_scale, a->strides, stream);
}

int apex_attn_fwd_varlen(const apex_attn_varlen_args* args, void* stream) {
  return forward_varlen(args, stream);
}

int apex_attn_fwd_noalloc(const void* q, const void* k, const void* v, void* o, float* lse,
                          int batch, int heads, int seqlen, int head_dim, int dtype, int causal,
                          float sm_scale, const long long* strides, void* stream) {
  return forward(true, q, k, v, o, lse, batch, heads, heads, seqlen, head_dim, dtype, causal, -1,
                 sm_scale, strides, stream);
}

int apex_attn_noalloc_status(int device, int* flags) {
  if (!flags) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  if (device < 0 || device >= kMaxDevices) return APEX_ATTN_ERR_NO_DEVICE;
  DeviceGuard guard(device);
  DeviceState* ds = nullptr;
  int rc = init_device_noalloc(device, &ds);
  if (rc != APEX_ATTN_OK) return rc;
  int word = 0;
  const int zero = 0;
  // Word 0 of the static scratch is the status word of the allocation-free launches.
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpyFromSymbol(&word, g_noalloc_scratch, sizeof(int), 0, cudaMemcpyDeviceToHost) != cudaSuccess ||
      cudaMemcpyToSymbol(g_noalloc_scratch, &zero, sizeof(int), 0, cudaMemcpyHostToDevice) != cudaSuccess) {
    (void)cudaGetLastError();
    return APEX_ATTN_ERR_CUDA;
  }
  *flags = word;
  return word ? APEX_ATTN_ERR_DEVICE_TIMEOUT : APEX_ATTN_OK;
}

int apex_attn_set_forward_kernel(int kind) {
  if (kind < 0 || kind > 2) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  g_fwd_kind.store(kind, std::memory_order_relaxed);
  return APEX_ATTN_OK;
}

int apex_attn_forward_kernel_for(int batch, int heads, int seq_len, int head_dim, int window,
                                 int packed, int num_sms) {
  if (batch <= 0 || heads <= 0 || seq_len <= 0 || num_sms <= 0 || window < -1 ||
      (head_dim != 64 && head_dim != 128 && head_dim != 256))
    return APEX_ATTN_ERR_INVALID_ARGUMENT;
  AttnParams p{};
  p.B = batch;
  p.H = heads;
  p.N = seq_len;
  p.window = window;
  static const int kPackedMarker = 0;
  p.cu_seqlens = packed ? &kPackedMarker : nullptr;
  const CUtensorMap map{};
  return use_tile_kernel(head_dim, p, packed ? nullptr : &map, num_sms) ? 2 : 1;
}

int apex_attn_num_sms_hint(int device) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    (void)cudaGetLastError();
    return APEX_ATTN_ERR_NO_DEVICE;
  }
  if (device < 0 || device >= count || device >= kMaxDevices) return APEX_ATTN_ERR_NO_DEVICE;
  DeviceState probe;
  std::lock_guard<std::mutex> lk(g_mu);
  const int rc = probe_device_locked(device, probe);
  return rc == APEX_ATTN_OK ? probe.num_sms : rc;
}

int apex_attn_device_status(int device, int* flags) {
  if (!flags) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(device);
  DeviceState* ds = nullptr;
  int rc = init_device(device, &ds);
  if (rc != APEX_ATTN_OK) return rc;
  int host[1] = {0};
  if (cudaDeviceSynchronize() != cudaSuccess) {
    (void)cudaGetLastError();
    return APEX_ATTN_ERR_CUDA;
  }
  if (cudaMemcpy(host, ds->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess ||
      cudaMemset(ds->status, 0, sizeof(int)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    (void)cudaGetLastError();
    return APEX_ATTN_ERR_CUDA;
  }
  *reinterpret_cast<volatile int*>(ds->host_flag) = 0;  // the device is idle: no kernel can set it now
  *flags = host[0];
  return host[0] ? APEX_ATTN_ERR_DEVICE_TIMEOUT : APEX_ATTN_OK;
}

int apex_attn_selftest_wait_timeout(int timeout_us, void* stream) {
  if (timeout_us <= 0 || timeout_us > 10 * 1000 * 1000) return APEX_ATTN_ERR_INVALID_ARGUMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return APEX_ATTN_ERR_NO_DEVICE;
  }
  DeviceState* ds = nullptr;
  int rc = init_device(dev, &ds);
  if (rc != APEX_ATTN_OK) return rc;
  wait_timeout_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      ds->status, ds->host_flag_dev, (unsigned long long)timeout_us * 1000ull);
  if (cudaGetLastError() != cudaSuccess) return APEX_ATTN_ERR_LAUNCH;
  return APEX_ATTN_OK;
}

}  // extern "C"

