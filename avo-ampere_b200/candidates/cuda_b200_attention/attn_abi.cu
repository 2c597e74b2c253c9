// C-ABI entry points of libavo_b200_attn.so (declared in include/avo_b200_attn.h).
//
// Host responsibilities: validate shapes/alignment the way the reference binding
// does (candidates/cuda_mma_attention/attention.cpp:13-21 and
// attention_kernel.cu:180-186: bf16, D == 128, matching shapes), check that the
// current device is a B200 (compute capability 10.0), build the TMA tensor maps and
// launch on the caller's stream.  The tensor-map encoder is fetched through
// cudaGetDriverEntryPoint so the library links no libcuda at build time and loads on
// machines without a GPU.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <mutex>

#include "attn_fwd.cuh"
#include "avo_b200_attn.h"

namespace avo_b200 {

// ---------------------------------------------------------------- LSE merge kernels
// One warp per (head, row): 32 lanes x 4 dims.
__global__ void lse_merge_kernel(float* __restrict__ acc_o, float* __restrict__ acc_lse,
                                 const __nv_bfloat16* __restrict__ part_o,
                                 const float* __restrict__ part_lse, int num_bh, int rows,
                                 long long ao_hs, long long al_hs, long long po_hs, long long pl_hs) {
  const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<long long>(num_bh) * rows) return;
  const long long h = gw / rows, r = gw % rows;
  float* lse_slot = acc_lse + h * al_hs + r;
  const float la = *lse_slot;
  const float lp = part_lse[h * pl_hs + r];
  const float lmax = fmaxf(la, lp);
  float wa = 0.f, wp = 0.f, lnew = -CUDART_INF_F;
  if (lmax != -CUDART_INF_F) {
    wa = expf(la - lmax);
    wp = expf(lp - lmax);
    const float sum = wa + wp;
    lnew = lmax + logf(sum);
    wa /= sum;
    wp /= sum;
  }
  float4* ap = reinterpret_cast<float4*>(acc_o + h * ao_hs + r * kHeadDim) + lane;
  const uint2 raw = *reinterpret_cast<const uint2*>(part_o + h * po_hs + r * kHeadDim + lane * 4);
  const float2 p01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 p23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  float4 a = *ap;
  if (wa == 0.f) {
    a = make_float4(p01.x * wp, p01.y * wp, p23.x * wp, p23.y * wp);
  } else {
    a = make_float4(a.x * wa + p01.x * wp, a.y * wa + p01.y * wp, a.z * wa + p23.x * wp,
                    a.w * wa + p23.y * wp);
  }
  *ap = a;
  __syncwarp();
  if (lane == 0) *lse_slot = lnew;
}

__global__ void acc_to_bf16_kernel(const float* __restrict__ acc_o, __nv_bfloat16* __restrict__ out,
                                   int num_bh, int rows, long long acc_hs, long long out_hs) {
  const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<long long>(num_bh) * rows) return;
  const long long h = gw / rows, r = gw % rows;
  const float4 a = reinterpret_cast<const float4*>(acc_o + h * acc_hs + r * kHeadDim)[lane];
  uint2 packed;
  packed.x = pack_bf16x2(a.x, a.y);
  packed.y = pack_bf16x2(a.z, a.w);
  *reinterpret_cast<uint2*>(out + h * out_hs + r * kHeadDim + lane * 4) = packed;
}

// One CTA waits on an mbarrier that is never completed; the bounded wait expires and
// reports through the status word.  Exercises the watchdog path without a fault.
__global__ void watchdog_selftest_kernel(int* status, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar_storage;
  __shared__ int abort_storage;
  if (threadIdx.x == 0) {
    mbar_init(smem_addr(&bar_storage), 1);
    abort_storage = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const Watch w{reinterpret_cast<volatile int*>(&abort_storage), status, limit_ns};
    (void)wait_phase(smem_addr(&bar_storage), 0, w);
  }
  __syncthreads();
}

// Evaluates the softmax's FMA-pipe exp2 (exp2_poly_x2) elementwise, two inputs per
// thread exactly as the kernel pairs them, so tests can hold it against CUDA's exp2f.
__global__ void exp2_poly_eval_kernel(const float* __restrict__ x, float* __restrict__ y, long long n) {
  const long long i = 2 * (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float x0 = x[i];
  const float x1 = i + 1 < n ? x[i + 1] : 0.f;
  float r0, r1;
  exp2_poly_x2(f2_pack(x0, x1), r0, r1);
  y[i] = r0;
  if (i + 1 < n) y[i + 1] = r1;
}

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

constexpr int kMaxDevices = 64;
std::mutex g_mu;
EncodeTiledFn g_encode = nullptr;
int g_device_state[kMaxDevices] = {};  // 0 unchecked, 1 ready, -1 not a B200
int g_sm_count[kMaxDevices] = {};      // multiprocessors, read once per device
int g_coop[kMaxDevices] = {};          // cooperative launch supported, read once per device

// Pipeline-wait limit (AVO_B200_WATCHDOG_MS, default 2 s).  It is wall-clock time
// (%globaltimer): on a GPU time-sliced between contexts (another process's work scheduled
// in between), a wait can also run out because this context was switched out that long;
// the launch then reports the watchdog bit although nothing was wrong.  Raise the limit on
// such shared GPUs.
unsigned long long watchdog_limit_ns() {
  static const unsigned long long limit = [] {
    const char* env = std::getenv("AVO_B200_WATCHDOG_MS");
    long long ms = env ? std::atoll(env) : 0;
    if (ms <= 0) ms = 2000;
    return static_cast<unsigned long long>(ms) * 1000000ull;
  }();
  return limit;
}

// Test hook, read once per process: AVO_B200_TEST_SKIP_LOAD=n makes each CTA's producer
// skip its n-th K/V copy (0-based, counted over the CTA's work items in order: K_0 V_0
// K_1 V_1 ... of its first item, then of its next), so the wait for it runs out and the
// launch exercises the kernel's watchdog abort path.  Unset (the default): -1, no skip.
int test_skip_load() {
  static const int skip = [] {
    const char* env = std::getenv("AVO_B200_TEST_SKIP_LOAD");
    return env ? std::atoi(env) : -1;
  }();
  return skip;
}

int resolve_encoder() {
  if (g_encode != nullptr) return AVO_B200_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult qres = cudaDriverEntryPointSymbolNotFound;
  const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qres);
  if (e != cudaSuccess || qres != cudaDriverEntryPointSuccess || fn == nullptr) {
    (void)cudaGetLastError();
    return AVO_B200_EDRIVER;
  }
  g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  return AVO_B200_OK;
}

// Checks the current device once (compute capability 10.0), raises the kernel's
// dynamic shared-memory limit on it and reads its multiprocessor count (optional out).
int prepare_device(int* sm_count = nullptr) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) {
    (void)cudaGetLastError();
    return AVO_B200_ENODEV;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  const int rc = resolve_encoder();
  if (rc != AVO_B200_OK) return rc;
  if (dev < kMaxDevices && g_device_state[dev] == 1) {
    if (sm_count != nullptr) *sm_count = g_sm_count[dev];
    return AVO_B200_OK;
  }
  if (dev < kMaxDevices && g_device_state[dev] == -1) return AVO_B200_ENODEV;
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return AVO_B200_ENODEV;
  }
  if (major != 10 || minor != 0) {
    if (dev < kMaxDevices) g_device_state[dev] = -1;
    return AVO_B200_ENODEV;
  }
  if (cudaFuncSetAttribute(attn_fwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
          cudaSuccess ||
      cudaFuncSetAttribute(attn_fwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
          cudaSuccess) {
    (void)cudaGetLastError();
    return AVO_B200_ELAUNCH;
  }
  // The kernel rebalances registers between warpgroups with setmaxnreg, which only
  // works out if the launch allocation is exactly the one the split was computed for;
  // otherwise an increase could wait forever.  Refuse to launch in that case.
  cudaFuncAttributes attr{}, attr_t{};
  if (cudaFuncGetAttributes(&attr, attn_fwd_kernel<false>) != cudaSuccess ||
      cudaFuncGetAttributes(&attr_t, attn_fwd_kernel<true>) != cudaSuccess) {
    (void)cudaGetLastError();
    return AVO_B200_ELAUNCH;
  }
  if (attr.numRegs != static_cast<int>(kRegsLaunch) || attr_t.numRegs != static_cast<int>(kRegsLaunch))
    return AVO_B200_EREGS;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    (void)cudaGetLastError();
    return AVO_B200_ENODEV;
  }
  int coop = 0;
  if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess) {
    (void)cudaGetLastError();
    coop = 0;
  }
  if (dev < kMaxDevices) {
    g_sm_count[dev] = sms;
    g_coop[dev] = coop != 0 ? 1 : 0;
    g_device_state[dev] = 1;
  }
  if (sm_count != nullptr) *sm_count = sms;
  return AVO_B200_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Whether the current device supports cooperative launches (all CTAs resident at once).
bool cooperative_ok() {
  int dev = -1, coop = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices && g_device_state[dev] == 1)
    return g_coop[dev] != 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return coop != 0;
}

// [heads, rows, 128] bf16 view with `head_stride` elements between heads; TMA box of
// 64 columns x 128 rows x 1 head, 128-byte swizzle.
int encode_rows(CUtensorMap* map, const void* base, int rows, int heads, long long head_stride) {
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(heads)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHeadDim) * 2,
                                 static_cast<cuuint64_t>(head_stride) * 2};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kBlockN), 1};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUresult r =
      g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
               estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? AVO_B200_OK : AVO_B200_ETENSORMAP;
}

// Scratch for split pieces inside a caller's workspace (zero-filled once by the caller; a
// launch that completes leaves every flag at 0 again): flags, then per slot m/l, then O.
struct SplitScratch {
  int* flags;
  float* ml;
  float* o;
};
constexpr size_t kFlagBytesPerCta = 2 * kQTiles * sizeof(int);
constexpr size_t kMlBytesPerCta = 2 * kQTiles * kSlotMl * sizeof(float);
constexpr size_t kOBytesPerCta = 2 * kQTiles * static_cast<size_t>(kSlotO) * sizeof(float);
size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
size_t workspace_bytes_for(int sms) {
  const size_t n = static_cast<size_t>(sms);
  return round_up(n * kFlagBytesPerCta, 256) + round_up(n * kMlBytesPerCta, 256) + n * kOBytesPerCta;
}
SplitScratch carve_workspace(void* ws, int sms) {
  const size_t n = static_cast<size_t>(sms);
  char* base = static_cast<char*>(ws);
  SplitScratch s;
  s.flags = reinterpret_cast<int*>(base);
  s.ml = reinterpret_cast<float*>(base + round_up(n * kFlagBytesPerCta, 256));
  s.o = reinterpret_cast<float*>(base + round_up(n * kFlagBytesPerCta, 256) + round_up(n * kMlBytesPerCta, 256));
  return s;
}

// Plans, with kTable's item lists, for the last few launch shapes (building the lists is
// a greedy pass per candidate group size: worth doing once per shape, not per launch).
struct PlanEntry {
  long long key[8];
  sched::Plan plan;
  TableParam<true> table;
};
constexpr int kPlanCache = 8;
PlanEntry g_plans[kPlanCache];
int g_plans_used = 0;
int g_plans_next = 0;

// Returns a copy (this thread's own) of the cached entry: another thread may replace the
// cache slot as soon as the lock is released.
const PlanEntry& cached_plan(int num_bh, int seq_q, int seq_kv, int causal, long long q_pos0, long long kv_pos0,
                             int sms, bool split_ok) {
  static thread_local PlanEntry mine;
  const long long key[8] = {num_bh, seq_q, seq_kv, causal ? 1 : 0, q_pos0, kv_pos0, sms, split_ok ? 1 : 0};
  std::lock_guard<std::mutex> lock(g_mu);
  for (int e = 0; e < g_plans_used; ++e) {
    bool same = true;
    for (int i = 0; i < 8; ++i) same = same && g_plans[e].key[i] == key[i];
    if (same) {
      // The 25 KB table is copied only for the plan that launches with it.
      mine.plan = g_plans[e].plan;
      if (mine.plan.mode == sched::kTable) mine.table = g_plans[e].table;
      return mine;
    }
  }
  PlanEntry& entry = g_plans[g_plans_next];
  g_plans_next = (g_plans_next + 1) % kPlanCache;
  if (g_plans_used < kPlanCache) ++g_plans_used;
  for (int i = 0; i < 8; ++i) entry.key[i] = key[i];
  entry.plan = sched::make_plan(num_bh, seq_q, seq_kv, causal, q_pos0, kv_pos0, sms, split_ok, &entry.table.t);
  mine = entry;
  return mine;
}

int launch_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int num_bh,
               int seq_q, int seq_kv, int head_dim, long long q_hs, long long kv_hs, long long o_hs,
               long long lse_hs, int causal, float scale, long long q_pos0, long long kv_pos0,
               int* status, void* stream, void* workspace = nullptr, size_t workspace_bytes = 0) {
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr) return AVO_B200_EINVAL;
  if (head_dim != kHeadDim || num_bh < 0 || seq_q < 0 || seq_kv < 0) return AVO_B200_EINVAL;
  if (!(scale > 0.f) || !std::isfinite(scale)) return AVO_B200_EINVAL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return AVO_B200_EINVAL;
  if (lse != nullptr && (reinterpret_cast<uintptr_t>(lse) & 3u) != 0) return AVO_B200_EINVAL;
  if (q_hs % 8 != 0 || kv_hs % 8 != 0 || o_hs % 8 != 0) return AVO_B200_EINVAL;
  if (q_hs < static_cast<long long>(seq_q) * kHeadDim || o_hs < static_cast<long long>(seq_q) * kHeadDim ||
      kv_hs < static_cast<long long>(seq_kv) * kHeadDim)
    return AVO_B200_EINVAL;
  if (lse != nullptr && lse_hs < seq_q) return AVO_B200_EINVAL;
  if (num_bh == 0 || seq_q == 0) return AVO_B200_OK;

  int sm_count = 0;
  int rc = prepare_device(&sm_count);
  if (rc != AVO_B200_OK) return rc;

  // Persistent grid: at most one CTA per multiprocessor (the kernel's shared memory admits
  // one), each walking its units of 256-row query blocks (schedule.cuh).
  const int num_q_blocks = (seq_q + kRowsPerCta - 1) / kRowsPerCta;
  const long long items = static_cast<long long>(num_bh) * num_q_blocks;
  if (items > INT_MAX) return AVO_B200_EINVAL;
  if (static_cast<long long>(num_bh) * ((seq_kv + kBlockN - 1) / kBlockN) * num_q_blocks > INT_MAX)
    return AVO_B200_EINVAL;
  const bool split_ok = workspace != nullptr && cooperative_ok();
  if (workspace != nullptr && workspace_bytes < workspace_bytes_for(sm_count)) return AVO_B200_EINVAL;
  if (workspace != nullptr && (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return AVO_B200_EINVAL;
  const PlanEntry& entry = cached_plan(num_bh, seq_q, seq_kv, causal, q_pos0, kv_pos0, sm_count, split_ok);
  const sched::Plan plan = entry.plan;
  const int grid = plan.grid;

  alignas(64) CUtensorMap tm_q, tm_k, tm_v;
  const int kv_rows = seq_kv > 0 ? seq_kv : 1;  // never read when seq_kv == 0
  if ((rc = encode_rows(&tm_q, q, seq_q, num_bh, q_hs)) != AVO_B200_OK) return rc;
  if ((rc = encode_rows(&tm_k, k, kv_rows, num_bh, kv_hs)) != AVO_B200_OK) return rc;
  if ((rc = encode_rows(&tm_v, v, kv_rows, num_bh, kv_hs)) != AVO_B200_OK) return rc;

  AttnParams p{};
  p.plan = plan;
  if (plan.mode != sched::kWaves) {
    const SplitScratch sc = carve_workspace(workspace, sm_count);
    p.part_flag = sc.flags;
    p.part_ml = sc.ml;
    p.part_o = sc.o;
  }
  p.lse = lse;
  p.o = o;
  p.o_head_stride = o_hs;
  p.o_sector_aligned = ((reinterpret_cast<uintptr_t>(o) & 31u) == 0 && o_hs % 16 == 0) ? 1 : 0;
  p.status = status;
  p.lse_head_stride = lse_hs;
  p.q_pos0 = q_pos0;
  p.kv_pos0 = kv_pos0;
  p.watchdog_ns = watchdog_limit_ns();
  p.test_skip_load = test_skip_load();
  p.seq_q = seq_q;
  p.seq_kv = seq_kv;
  p.num_bh = num_bh;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;

  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (plan.mode == sched::kWaves) {
    // Programmatic dependent launch: this launch's CTAs may start their set-up on free
    // multiprocessors while the previous work in the stream finishes (the kernel waits for
    // it before touching global memory).  Measured on B200: ~1.3 us less per back-to-back
    // launch of small problems.  The table plan keeps plain ordering (it measured 2 % more
    // cycles with it: two 25 KB parameter blocks then compete in the constant cache), as
    // does the split plan's cooperative launch.
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, attn_fwd_kernel<false>, tm_q, tm_k, tm_v, p, TableParam<false>{0}) != cudaSuccess) {
      (void)cudaGetLastError();
      return AVO_B200_ELAUNCH;
    }
  } else if (plan.mode == sched::kTable) {
    attn_fwd_kernel<true><<<static_cast<unsigned>(grid), kThreads, kSmemBytes, st>>>(tm_q, tm_k, tm_v, p,
                                                                                      entry.table);
  } else {
    // Split pieces: a CTA that merges an item waits for its neighbours' continuation
    // pieces, so every CTA must be resident at once; a cooperative launch guarantees it
    // (or fails to launch).
    TableParam<false> none{0};
    void* args[] = {&tm_q, &tm_k, &tm_v, &p, &none};
    if (cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(attn_fwd_kernel<false>), dim3(grid),
                                    dim3(kThreads), args, kSmemBytes, st) != cudaSuccess) {
      (void)cudaGetLastError();
      return AVO_B200_ELAUNCH;
    }
  }
  if (cudaGetLastError() != cudaSuccess) return AVO_B200_ELAUNCH;
  return AVO_B200_OK;
}

}  // namespace
}  // namespace avo_b200

using namespace avo_b200;

extern "C" int avo_b200_abi_version(void) { return 1; }

extern "C" const char* avo_b200_strerror(int code) {
  switch (code) {
    case AVO_B200_OK: return "ok";
    case AVO_B200_EINVAL: return "invalid argument";
    case AVO_B200_ENODEV: return "current CUDA device is not a B200 (compute capability 10.0)";
    case AVO_B200_ELAUNCH: return "CUDA launch error";
    case AVO_B200_ETENSORMAP: return "tensor map encoding failed";
    case AVO_B200_EDRIVER: return "driver entry point cuTensorMapEncodeTiled unavailable";
    case AVO_B200_EREGS:
      return "attention kernel built with an unexpected register count (the setmaxnreg split needs 168 per "
             "thread at launch); rebuild the library";
    case AVO_B200_ETOOBIG:
      return "problem too large for the no-allocation entry point (batch*heads*seq > 16384 rows)";
    default: return "unknown error";
  }
}

extern "C" int avo_b200_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                                 int batch, int heads, int seq, int head_dim, int causal,
                                 float softmax_scale, int* status_dev, void* stream) {
  if (batch < 0 || heads < 0 || seq < 0) return AVO_B200_EINVAL;
  const long long bh = static_cast<long long>(batch) * heads;
  if (bh > INT_MAX) return AVO_B200_EINVAL;
  const long long hs = static_cast<long long>(seq) * kHeadDim;
  return launch_fwd(q, k, v, o, lse, static_cast<int>(bh), seq, seq, head_dim, hs, hs, hs, seq, causal,
                    softmax_scale, 0, 0, status_dev, stream);
}

extern "C" int avo_b200_attn_workspace_size(size_t* bytes) {
  if (bytes == nullptr) return AVO_B200_EINVAL;
  int sm_count = 0;
  const int rc = prepare_device(&sm_count);
  if (rc != AVO_B200_OK) return rc;
  *bytes = workspace_bytes_for(sm_count);
  return AVO_B200_OK;
}

extern "C" int avo_b200_attn_fwd_ws(const void* q, const void* k, const void* v, void* o, float* lse, int batch,
                                    int heads, int seq, int head_dim, int causal, float softmax_scale,
                                    void* workspace, size_t workspace_bytes, int* status_dev, void* stream) {
  if (batch < 0 || heads < 0 || seq < 0) return AVO_B200_EINVAL;
  const long long bh = static_cast<long long>(batch) * heads;
  if (bh > INT_MAX) return AVO_B200_EINVAL;
  const long long hs = static_cast<long long>(seq) * kHeadDim;
  return launch_fwd(q, k, v, o, lse, static_cast<int>(bh), seq, seq, head_dim, hs, hs, hs, seq, causal,
                    softmax_scale, 0, 0, status_dev, stream, workspace, workspace_bytes);
}

extern "C" int avo_b200_schedule_units(int num_bh, int seq_q, int seq_kv, int causal, long long q_pos0,
                                       long long kv_pos0, int sm_count, int split, int* plan_out,
                                       int* units, int max_units, int* counts) {
  if (num_bh < 0 || seq_q < 0 || seq_kv < 0 || sm_count <= 0 || plan_out == nullptr || max_units < 0)
    return AVO_B200_EINVAL;
  static thread_local sched::Table table;
  const sched::Plan plan =
      sched::make_plan(num_bh, seq_q, seq_kv, causal, q_pos0, kv_pos0, sm_count, split != 0, &table);
  plan_out[0] = plan.mode;
  plan_out[1] = plan.grid;
  plan_out[2] = plan.mode == sched::kTable ? plan.group_pairs : plan.run_min;
  plan_out[3] = plan.wave_items;
  if (units == nullptr || counts == nullptr) return AVO_B200_OK;
  for (int c = 0; c < plan.grid; ++c) {
    sched::Walker walk(plan, c, &table);
    sched::Unit u;
    int n = 0;
    while (walk.next(u)) {
      if (n < max_units) {
        int* e = units + (static_cast<long long>(c) * max_units + n) * 8;
        e[0] = u.bh; e[1] = u.q0; e[2] = u.t0; e[3] = u.t1; e[4] = u.kind; e[5] = u.seg;
        e[6] = u.cont_lo; e[7] = u.cont_hi;
      }
      ++n;
    }
    counts[c] = n;
  }
  return AVO_B200_OK;
}

extern "C" int avo_b200_attn_fwd_block(const void* q, const void* k, const void* v, void* o, float* lse,
                                       int num_bh, int seq_q, int seq_kv, int head_dim,
                                       long long q_head_stride, long long kv_head_stride,
                                       long long o_head_stride, long long lse_head_stride, int causal,
                                       float softmax_scale, long long q_pos0, long long kv_pos0,
                                       int* status_dev, void* stream) {
  return launch_fwd(q, k, v, o, lse, num_bh, seq_q, seq_kv, head_dim, q_head_stride, kv_head_stride,
                    o_head_stride, lse_head_stride, causal, softmax_scale, q_pos0, kv_pos0, status_dev,
                    stream);
}

extern "C" int avo_b200_lse_merge(float* acc_o, float* acc_lse, const void* part_o, const float* part_lse,
                                  int num_bh, int rows, int head_dim, long long acc_o_head_stride,
                                  long long acc_lse_head_stride, long long part_o_head_stride,
                                  long long part_lse_head_stride, void* stream) {
  if (acc_o == nullptr || acc_lse == nullptr || part_o == nullptr || part_lse == nullptr)
    return AVO_B200_EINVAL;
  if (head_dim != kHeadDim || num_bh < 0 || rows < 0) return AVO_B200_EINVAL;
  const long long row_elems = static_cast<long long>(rows) * kHeadDim;
  if (acc_o_head_stride % 4 != 0 || part_o_head_stride % 4 != 0 || acc_o_head_stride < row_elems ||
      part_o_head_stride < row_elems || acc_lse_head_stride < rows || part_lse_head_stride < rows)
    return AVO_B200_EINVAL;
  if (!aligned16(acc_o) || (reinterpret_cast<uintptr_t>(part_o) & 7u) != 0) return AVO_B200_EINVAL;
  const long long warps = static_cast<long long>(num_bh) * rows;
  if (warps == 0) return AVO_B200_OK;
  const long long blocks = (warps * 32 + 255) / 256;
  if (blocks > INT_MAX) return AVO_B200_EINVAL;
  lse_merge_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      acc_o, acc_lse, reinterpret_cast<const __nv_bfloat16*>(part_o), part_lse, num_bh, rows,
      acc_o_head_stride, acc_lse_head_stride, part_o_head_stride, part_lse_head_stride);
  return cudaGetLastError() == cudaSuccess ? AVO_B200_OK : AVO_B200_ELAUNCH;
}

extern "C" int avo_b200_acc_to_bf16(const float* acc_o, void* out, int num_bh, int rows, int head_dim,
                                    long long acc_head_stride, long long out_head_stride, void* stream) {
  if (acc_o == nullptr || out == nullptr || head_dim != kHeadDim || num_bh < 0 || rows < 0)
    return AVO_B200_EINVAL;
  const long long row_elems = static_cast<long long>(rows) * kHeadDim;
  if (acc_head_stride % 4 != 0 || out_head_stride % 4 != 0 || acc_head_stride < row_elems ||
      out_head_stride < row_elems)
    return AVO_B200_EINVAL;
  if (!aligned16(acc_o) || (reinterpret_cast<uintptr_t>(out) & 7u) != 0) return AVO_B200_EINVAL;
  const long long warps = static_cast<long long>(num_bh) * rows;
  if (warps == 0) return AVO_B200_OK;
  const long long blocks = (warps * 32 + 255) / 256;
  if (blocks > INT_MAX) return AVO_B200_EINVAL;
  acc_to_bf16_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      acc_o, reinterpret_cast<__nv_bfloat16*>(out), num_bh, rows, acc_head_stride, out_head_stride);
  return cudaGetLastError() == cudaSuccess ? AVO_B200_OK : AVO_B200_ELAUNCH;
}

extern "C" int avo_b200_watchdog_selftest(int timeout_us, int* status_dev, void* stream) {
  if (status_dev == nullptr || timeout_us <= 0 || timeout_us > 10000000) return AVO_B200_EINVAL;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return AVO_B200_ENODEV;
  }
  watchdog_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      status_dev, static_cast<unsigned long long>(timeout_us) * 1000ull);
  return cudaGetLastError() == cudaSuccess ? AVO_B200_OK : AVO_B200_ELAUNCH;
}

extern "C" int avo_b200_exp2_poly_eval(const float* x, float* y, long long n, void* stream) {
  if (x == nullptr || y == nullptr || n < 0) return AVO_B200_EINVAL;
  if (n == 0) return AVO_B200_OK;
  const long long blocks = ((n + 1) / 2 + 255) / 256;
  if (blocks > INT_MAX) return AVO_B200_EINVAL;
  exp2_poly_eval_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
  return cudaGetLastError() == cudaSuccess ? AVO_B200_OK : AVO_B200_ELAUNCH;
}

// ---------------------------------------------------------------- no-allocation split path
// Scratch of avo_b200_attn_fwd_split_noalloc, held statically on every device the library
// runs on: a running fp32 accumulator (O and LSE) and one bf16/fp32 partial, each for up to
// AVO_B200_NOALLOC_MAX_ROWS rows of 128 values.  About 12.1 MiB per device.
static __device__ __align__(256) float g_noalloc_acc_o[AVO_B200_NOALLOC_MAX_ROWS * kHeadDim];
static __device__ __align__(256) float g_noalloc_acc_lse[AVO_B200_NOALLOC_MAX_ROWS];
static __device__ __align__(256) __nv_bfloat16 g_noalloc_part_o[AVO_B200_NOALLOC_MAX_ROWS * kHeadDim];
static __device__ __align__(256) float g_noalloc_part_lse[AVO_B200_NOALLOC_MAX_ROWS];

namespace avo_b200 {
namespace noalloc {

__global__ void fill_f32_kernel(float* __restrict__ p, float value, long long n) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) p[i] = value;
}

struct NoAllocScratch {
  float* acc_o;
  float* acc_lse;
  void* part_o;
  float* part_lse;
};

// Device addresses of the static scratch, resolved with cudaGetSymbolAddress once per
// device (the call needs the current device's context and costs a driver round trip).
int noalloc_scratch(NoAllocScratch* out) {
  static NoAllocScratch cache[kMaxDevices];
  static bool ready[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    (void)cudaGetLastError();
    return AVO_B200_ENODEV;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (!ready[dev]) {
    NoAllocScratch s{};
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&s.acc_o), g_noalloc_acc_o) != cudaSuccess ||
        cudaGetSymbolAddress(reinterpret_cast<void**>(&s.acc_lse), g_noalloc_acc_lse) != cudaSuccess ||
        cudaGetSymbolAddress(&s.part_o, g_noalloc_part_o) != cudaSuccess ||
        cudaGetSymbolAddress(reinterpret_cast<void**>(&s.part_lse), g_noalloc_part_lse) != cudaSuccess) {
      (void)cudaGetLastError();
      return AVO_B200_ELAUNCH;
    }
    cache[dev] = s;
    ready[dev] = true;
  }
  *out = cache[dev];
  return AVO_B200_OK;
}

}  // namespace noalloc
}  // namespace avo_b200

extern "C" int avo_b200_attn_fwd_split_noalloc(const void* q, const void* k, const void* v, void* o, float* lse,
                                                int batch, int heads, int seq, int head_dim, int causal,
                                                float softmax_scale, int n_splits, int* status_dev,
                                                void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr) return AVO_B200_EINVAL;
  if (batch < 0 || heads < 0 || seq < 0 || head_dim != kHeadDim) return AVO_B200_EINVAL;
  if (n_splits < 1 || n_splits > AVO_B200_NOALLOC_MAX_SPLITS) return AVO_B200_EINVAL;
  if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale)) return AVO_B200_EINVAL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return AVO_B200_EINVAL;
  if (lse != nullptr && (reinterpret_cast<uintptr_t>(lse) & 3u) != 0) return AVO_B200_EINVAL;
  // Size check before any product that could overflow: batch, heads and seq are each
  // non-negative ints, so batch * heads fits in 64 bits, and the row count is only formed
  // once it is known to stay within the scratch.
  const long long bh = static_cast<long long>(batch) * heads;
  if (bh > AVO_B200_NOALLOC_MAX_ROWS || (seq > 0 && bh > AVO_B200_NOALLOC_MAX_ROWS / seq))
    return AVO_B200_ETOOBIG;
  const long long rows = bh * seq;
  if (rows == 0) return AVO_B200_OK;

  int rc = prepare_device();
  if (rc != AVO_B200_OK) return rc;
  noalloc::NoAllocScratch s;
  if ((rc = noalloc::noalloc_scratch(&s)) != AVO_B200_OK) return rc;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);

  // The accumulator starts empty: LSE = -inf (its O is then never read, see lse_merge).
  noalloc::fill_f32_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, st>>>(s.acc_lse, -INFINITY, rows);
  if (cudaGetLastError() != cudaSuccess) return AVO_B200_ELAUNCH;

  const int n_kv_tiles = (seq + kBlockN - 1) / kBlockN;
  const int tiles_per_split = (n_kv_tiles + n_splits - 1) / n_splits;
  const long long hs = static_cast<long long>(seq) * kHeadDim;
  const int nbh = static_cast<int>(bh);
  for (int sp = 0; sp < n_splits; ++sp) {
    const long long k0 = static_cast<long long>(sp) * tiles_per_split * kBlockN;
    if (k0 >= seq) break;
    const int kv_len = static_cast<int>(std::min<long long>(seq - k0, static_cast<long long>(tiles_per_split) * kBlockN));
    const size_t off = static_cast<size_t>(k0) * kHeadDim * sizeof(__nv_bfloat16);
    // Keys [k0, k0 + kv_len) of every head; the causal mask uses their true positions.
    rc = launch_fwd(q, static_cast<const char*>(k) + off, static_cast<const char*>(v) + off, s.part_o, s.part_lse,
                    nbh, seq, kv_len, head_dim, hs, hs, hs, seq, causal, softmax_scale, 0, k0, status_dev, stream);
    if (rc != AVO_B200_OK) return rc;
    rc = avo_b200_lse_merge(s.acc_o, s.acc_lse, s.part_o, s.part_lse, nbh, seq, head_dim, hs, seq, hs, seq, stream);
    if (rc != AVO_B200_OK) return rc;
  }
  rc = avo_b200_acc_to_bf16(s.acc_o, o, nbh, seq, head_dim, hs, hs, stream);
  if (rc != AVO_B200_OK) return rc;
  if (lse != nullptr &&
      cudaMemcpyAsync(lse, s.acc_lse, static_cast<size_t>(rows) * sizeof(float), cudaMemcpyDeviceToDevice, st) !=
          cudaSuccess) {
    (void)cudaGetLastError();
    return AVO_B200_ELAUNCH;
  }
  return AVO_B200_OK;
}
