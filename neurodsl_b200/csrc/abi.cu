// abi.cu — extern "C" entry points of libneurodsl_b200.so.
//
// Validates every argument on the host before any launch (shape, alignment,
// dtype, device), converts failures to ND_ERR_* status codes with a message
// in nd_last_error_string(), and forwards to the kernel launchers.  The
// reference reports failures with error("❌ ...") (e.g. src/dispatch.jl:8,583);
// the host wrappers turn a non-zero status back into an exception.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "../../include/neurodsl_b200.h"
#include "flash_fwd.h"
#include "gemm.h"
#include "kv_decode.h"
#include "launch.cuh"
#include "elementwise.h"
#include "layernorm.h"
#include "model_ops.h"
#include "tp_comm.h"
#include "tma.h"

namespace {
// Device error word: one int per device (a __device__ variable exists once
// per device that loads the library).
__device__ int g_device_error = 0;
}  // namespace

namespace nd {
int* device_error_word() {
  // The address is cached per host thread and device, together with the id
  // of the context it belongs to (a context torn down and created again
  // reloads the variable, possibly elsewhere); a per-thread cache needs no
  // lock on this per-launch path.
  thread_local int* cached[64] = {};
  thread_local unsigned long long cached_ctx[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  const unsigned long long ctx = current_context_id();
  if (cached[dev] == nullptr || cached_ctx[dev] != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<int*>(p);
    cached_ctx[dev] = ctx;
  }
  return cached[dev];
}
namespace {
thread_local bool t_pdl = false;
thread_local int t_sm_limit = 0;
}  // namespace
bool pdl_enabled() { return t_pdl; }
void set_pdl_enabled(bool on) { t_pdl = on; }
int sm_limit() { return t_sm_limit; }
void set_sm_limit(int n) { t_sm_limit = n; }
int current_sm_count() {
  static std::atomic<int> counts[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = counts[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      return 148;
    counts[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}
}  // namespace nd

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_err[0] = '\0';
  return ND_OK;
}

int cuda_fail(cudaError_t e, const char* where, const char* extra = nullptr) {
  return fail(ND_ERR_CUDA, "%s: %s%s%s", where, cudaGetErrorString(e), extra ? " — " : "",
              extra ? extra : "");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr int kMaxDevices = 64;
int g_cc_major[kMaxDevices];  // 0 = unknown

// Checks that the current device is sm_100; caches the answer per device.
int check_current_device(int* dev_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(ND_ERR_DEVICE, "device index %d out of range", dev);
  int major = __atomic_load_n(&g_cc_major[dev], __ATOMIC_ACQUIRE);
  if (major == 0) {
    int minor = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    if (major != 10 || minor != 0)
      return fail(ND_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                  major, minor);
    __atomic_store_n(&g_cc_major[dev], major, __ATOMIC_RELEASE);
  }
  if (dev_out) *dev_out = dev;
  return ND_OK;
}

// Library-owned decode scratch, one buffer per device, grown on demand and
// zero-filled when (re)allocated.  Growth synchronises the device, so a
// caller that captures decode into a CUDA graph makes one uncaptured call of
// the largest size first.  The zero fill runs on the caller's stream and is
// waited for before the call returns, so a kernel on any stream that uses the
// buffer afterwards sees the tickets at zero.
struct OwnedWorkspace {
  void* ptr = nullptr;
  size_t bytes = 0;
};
OwnedWorkspace g_ws[kMaxDevices];
std::mutex g_ws_mu;

int owned_workspace(int dev, size_t need, cudaStream_t stream, void** out) {
  std::lock_guard<std::mutex> lk(g_ws_mu);
  OwnedWorkspace& w = g_ws[dev];
  if (w.bytes < need) {
    if (w.ptr) {
      cudaError_t e = cudaFree(w.ptr);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFree (decode workspace)");
      w.ptr = nullptr;
      w.bytes = 0;
    }
    size_t sz = need < (1u << 20) ? (1u << 20) : need;
    cudaError_t e = cudaMalloc(&w.ptr, sz);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (decode workspace)");
    e = cudaMemsetAsync(w.ptr, 0, sz, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync (decode workspace)");
    w.bytes = sz;
  }
  *out = w.ptr;
  return ND_OK;
}

// ---- 2-D layout conversion kernel (32x32 tiles through shared memory) ------
template <typename TS, typename TD>
__device__ __forceinline__ TD cvt(TS v);
template <> __device__ __forceinline__ float cvt<float, float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 cvt<float, __nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ float cvt<__nv_bfloat16, float>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16, __nv_bfloat16>(__nv_bfloat16 v) { return v; }

// dst rows are ld_dst elements apart; columns [cols, ld_dst) are written as
// zeros (an inner dimension padded to the GEMM's 16-byte rows in the same pass).
template <typename TS, typename TD, bool kColMajor>
__global__ void convert_kernel(const TS* __restrict__ src, TD* __restrict__ dst, int rows,
                               int cols, int ld_dst) {
  __shared__ TS tile[32][33];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  if (kColMajor) {
    // read coalesced along rows of the column-major source
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
      const int c = c0 + i, r = r0 + threadIdx.x;
      if (r < rows && c < cols) tile[threadIdx.x][i] = src[static_cast<size_t>(c) * rows + r];
    }
  } else {
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
      const int r = r0 + i, c = c0 + threadIdx.x;
      if (r < rows && c < cols) tile[i][threadIdx.x] = src[static_cast<size_t>(r) * cols + c];
    }
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < ld_dst)
      dst[static_cast<size_t>(r) * ld_dst + c] =
          c < cols ? cvt<TS, TD>(tile[i][threadIdx.x]) : cvt<float, TD>(0.f);
  }
}

template <typename TS, typename TD>
cudaError_t launch_convert(cudaStream_t st, const void* src, void* dst, int rows, int cols,
                           bool col_major, int ld_dst) {
  dim3 block(32, 8), grid((ld_dst + 31) / 32, (rows + 31) / 32);
  if (col_major)
    convert_kernel<TS, TD, true><<<grid, block, 0, st>>>(static_cast<const TS*>(src), static_cast<TD*>(dst), rows, cols, ld_dst);
  else
    convert_kernel<TS, TD, false><<<grid, block, 0, st>>>(static_cast<const TS*>(src), static_cast<TD*>(dst), rows, cols, ld_dst);
  return cudaGetLastError();
}

bool valid_dtype(int t) { return t == ND_F32 || t == ND_BF16; }

}  // namespace

static int kv_decode_impl(const char* fn, void* stream, const void* q, const void* k_new,
                          const void* v_new, long long qkv_ld, void* k_cache, void* v_cache,
                          void* out, int o_dtype, float* lse, int B, int H, int L, int L_max,
                          int D, float scale, void* workspace, size_t workspace_bytes) {
  if (B < 0 || H < 0) return fail(ND_ERR_INVALID_ARG, "%s: negative size", fn);
  if (D != 64) return fail(ND_ERR_UNSUPPORTED, "%s: head_dim %d not supported (64 only)", fn, D);
  if (L < 1 || L > L_max)
    return fail(ND_ERR_SHAPE, "%s: need 1 <= L <= L_max (L=%d, L_max=%d)", fn, L, L_max);
  if (!valid_dtype(o_dtype)) return fail(ND_ERR_UNSUPPORTED, "%s: bad o_dtype %d", fn, o_dtype);
  if ((k_new == nullptr) != (v_new == nullptr))
    return fail(ND_ERR_INVALID_ARG, "%s: k_new and v_new must both be given or both NULL", fn);
  if (static_cast<long long>(B) * H > 65535)
    return fail(ND_ERR_SHAPE, "%s: B*H = %lld exceeds 65535", fn, static_cast<long long>(B) * H);
  if (B == 0 || H == 0) return ok();
  if (!q || !k_cache || !v_cache || !out) return fail(ND_ERR_INVALID_ARG, "%s: null tensor pointer", fn);
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out) ||
      (k_new && (!aligned16(k_new) || !aligned16(v_new))))
    return fail(ND_ERR_ALIGNMENT, "%s: tensors must be 16-byte aligned", fn);
  int dev = 0;
  int rc = check_current_device(&dev);
  if (rc) return rc;
  const size_t need = nd::kv_decode_workspace_bytes(B, H, L);
  void* ws = workspace;
  if (need > 0) {
    if (ws == nullptr) {
      rc = owned_workspace(dev, need, static_cast<cudaStream_t>(stream), &ws);
      if (rc) return rc;
    } else if (workspace_bytes < need) {
      return fail(ND_ERR_WORKSPACE, "%s: workspace %zu bytes < %zu needed", fn, workspace_bytes, need);
    } else if (!aligned16(ws)) {
      return fail(ND_ERR_ALIGNMENT, "%s: workspace must be 16-byte aligned", fn);
    }
  }
  cudaError_t e = nd::launch_kv_decode(
      static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(q),
      static_cast<const __nv_bfloat16*>(k_new), static_cast<const __nv_bfloat16*>(v_new),
      static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), out,
      o_dtype == ND_F32, lse, B, H, L, L_max, scale, ws, qkv_ld);
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return ok();
}



extern "C" {

__attribute__((visibility("default"))) int nd_version(void) { return 100; }

__attribute__((visibility("default"))) const char* nd_last_error_string(void) { return g_err; }

__attribute__((visibility("default"))) int nd_device_check(int device) {
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (device != prev) {
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  }
  int rc = check_current_device(nullptr);
  if (device != prev) cudaSetDevice(prev);
  return rc == ND_OK ? ok() : rc;
}

__attribute__((visibility("default"))) int nd_device_error(int* code) {
  if (code == nullptr) return fail(ND_ERR_INVALID_ARG, "nd_device_error: code is NULL");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  int zero = 0;
  e = cudaMemcpyFromSymbol(code, g_device_error, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "device error word");
  return ok();
}

namespace {
// Shared argument checks and launch of the two prefill entry points.
// The stride of a dimension of extent 1 is never applied; give it a value
// that passes the layout checks (head-major, batch outermost).
void normalize_unit_strides(long long (&s)[3], int S, int H, int B) {
  if (H == 1) s[1] = s[0] * (S > 0 ? S : 1);
  if (B == 1) {
    const long long a = s[0] * (S > 0 ? S : 1), b = s[1] * (H > 0 ? H : 1);
    s[2] = a > b ? a : b;
  }
}

int flash_attn_common(const char* fn, void* stream, const void* Q, const void* K, const void* V,
                      void* O, int o_dtype, float* lse, float* row_max, int B, int H, int Sq,
                      int Sk, int D, float scale, int causal, nd::FlashStrides st) {
  normalize_unit_strides(st.q, Sq, H, B);
  normalize_unit_strides(st.o, Sq, H, B);
  normalize_unit_strides(st.k, Sk, H, B);
  normalize_unit_strides(st.v, Sk, H, B);
  if (B < 0 || H < 0 || Sq < 0 || Sk < 0)
    return fail(ND_ERR_INVALID_ARG, "%s: negative size (B=%d H=%d Sq=%d Sk=%d)", fn, B, H, Sq, Sk);
  if (D != 64) return fail(ND_ERR_UNSUPPORTED, "%s: head_dim %d not supported (64 only)", fn, D);
  if (!valid_dtype(o_dtype)) return fail(ND_ERR_UNSUPPORTED, "%s: bad o_dtype %d", fn, o_dtype);
  if (causal && Sq != Sk)
    return fail(ND_ERR_SHAPE, "%s: causal attention needs Sq == Sk (got %d, %d)", fn, Sq, Sk);
  if (!causal && Sk == 0 && Sq > 0)
    return fail(ND_ERR_SHAPE, "%s: no keys (Sk = 0) for %d queries", fn, Sq);
  if (static_cast<long long>(B) * H * ((Sq + 127) / 128) > 0x7fffffffLL)
    return fail(ND_ERR_SHAPE, "%s: grid too large", fn);
  if (B == 0 || H == 0 || Sq == 0) return ok();
  if (!Q || !K || !V || !O) return fail(ND_ERR_INVALID_ARG, "%s: null tensor pointer", fn);
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O))
    return fail(ND_ERR_ALIGNMENT, "%s: Q/K/V/O must be 16-byte aligned", fn);
  const long long* all[4] = {st.q, st.k, st.v, st.o};
  const char* names = "QKVO";
  for (int t = 0; t < 4; ++t) {
    for (int i = 0; i < 3; ++i) {
      const long long x = all[t][i];
      if (x <= 0 || x % 8 != 0 || x >= (1LL << 38))
        return fail(ND_ERR_SHAPE, "%s: %c stride[%d] = %lld must be a positive multiple of 8 elements below 2^38",
                    fn, names[t], i, x);
    }
    if (t < 3 && all[t][2] < (all[t][0] > all[t][1] ? all[t][0] : all[t][1]))
      return fail(ND_ERR_SHAPE, "%s: %c batch stride must be the outermost (>= row and head strides)", fn, names[t]);
  }
  if ((st.k[1] < st.k[0]) != (st.v[1] < st.v[0]))
    return fail(ND_ERR_SHAPE, "%s: K and V must share one layout (both head-major or both token-major)", fn);
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  const char* msg = nullptr;
  cudaError_t e = nd::launch_flash_fwd(static_cast<cudaStream_t>(stream),
                                       static_cast<const __nv_bfloat16*>(Q),
                                       static_cast<const __nv_bfloat16*>(K),
                                       static_cast<const __nv_bfloat16*>(V), O, o_dtype == ND_F32,
                                       lse, row_max, B, H, Sq, Sk, scale, causal != 0, st, &msg);
  if (e != cudaSuccess) return cuda_fail(e, fn, msg);
  return ok();
}
}  // namespace

__attribute__((visibility("default"))) int nd_flash_attn_fwd(void* stream, const void* Q,
                                                             const void* K, const void* V, void* O,
                                                             int o_dtype, float* lse,
                                                             float* row_max, int B, int H, int Sq,
                                                             int Sk, int D, float scale,
                                                             int causal) {
  return flash_attn_common("nd_flash_attn_fwd", stream, Q, K, V, O, o_dtype, lse, row_max, B, H,
                           Sq, Sk, D, scale, causal,
                           nd::flash_head_major_strides(H < 1 ? 1 : H, Sq, Sk));
}

__attribute__((visibility("default"))) int nd_flash_attn_fwd_strided(
    void* stream, const void* Q, const int64_t* q_strides, const void* K, const int64_t* k_strides,
    const void* V, const int64_t* v_strides, void* O, const int64_t* o_strides, int o_dtype,
    float* lse, float* row_max, int B, int H, int Sq, int Sk, int D, float scale, int causal) {
  if (!q_strides || !k_strides || !v_strides || !o_strides)
    return fail(ND_ERR_INVALID_ARG, "nd_flash_attn_fwd_strided: null stride array");
  nd::FlashStrides st;
  for (int i = 0; i < 3; ++i) {
    st.q[i] = q_strides[i];
    st.k[i] = k_strides[i];
    st.v[i] = v_strides[i];
    st.o[i] = o_strides[i];
  }
  return flash_attn_common("nd_flash_attn_fwd_strided", stream, Q, K, V, O, o_dtype, lse, row_max,
                           B, H, Sq, Sk, D, scale, causal, st);
}

__attribute__((visibility("default"))) int nd_kv_decode_workspace_size(int B, int H, int L, int D,
                                                                       size_t* bytes) {
  if (!bytes) return fail(ND_ERR_INVALID_ARG, "nd_kv_decode_workspace_size: bytes is NULL");
  if (B < 0 || H < 0 || L < 0) return fail(ND_ERR_INVALID_ARG, "nd_kv_decode_workspace_size: negative size");
  if (D != 64) return fail(ND_ERR_UNSUPPORTED, "nd_kv_decode_workspace_size: head_dim %d not supported", D);
  *bytes = nd::kv_decode_workspace_bytes(B, H, L);
  return ok();
}

__attribute__((visibility("default"))) int nd_kv_decode_attn(
    void* stream, const void* q, const void* k_new, const void* v_new, void* k_cache,
    void* v_cache, void* out, int o_dtype, float* lse, int B, int H, int L, int L_max, int D,
    float scale, void* workspace, size_t workspace_bytes) {
  return kv_decode_impl("nd_kv_decode_attn", stream, q, k_new, v_new, 0, k_cache, v_cache, out,
                        o_dtype, lse, B, H, L, L_max, D, scale, workspace, workspace_bytes);
}

// Decode attention straight from a fused QKV projection: row b of qkv holds
// q, then k_new, then v_new (H*D values each), rows qkv_ld elements apart.
__attribute__((visibility("default"))) int nd_kv_decode_attn_qkv(
    void* stream, const void* qkv, int64_t qkv_ld, void* k_cache, void* v_cache, void* out,
    int o_dtype, float* lse, int B, int H, int L, int L_max, int D, float scale, void* workspace,
    size_t workspace_bytes) {
  if (B < 0 || H < 0) return fail(ND_ERR_INVALID_ARG, "nd_kv_decode_attn_qkv: negative size");
  if (D != 64)
    return fail(ND_ERR_UNSUPPORTED, "nd_kv_decode_attn_qkv: head_dim %d not supported (64 only)", D);
  if (B == 0 || H == 0) return ok();
  if (qkv == nullptr) return fail(ND_ERR_INVALID_ARG, "nd_kv_decode_attn_qkv: qkv is NULL");
  if (qkv_ld < 3LL * H * D || qkv_ld % 8 != 0)
    return fail(ND_ERR_SHAPE,
                "nd_kv_decode_attn_qkv: row stride %lld must be >= 3*H*D = %lld and a multiple of 8",
                static_cast<long long>(qkv_ld), 3LL * H * D);
  const char* base = static_cast<const char*>(qkv);
  const size_t block = static_cast<size_t>(H) * D * sizeof(__nv_bfloat16);
  return kv_decode_impl("nd_kv_decode_attn_qkv", stream, qkv, base + block, base + 2 * block,
                        static_cast<long long>(qkv_ld), k_cache, v_cache, out, o_dtype, lse, B, H,
                        L, L_max, D, scale, workspace, workspace_bytes);
}

// Programmatic dependent launch for this host thread's later launches of the
// decode-step kernels (see launch.cuh for the rule those kernels follow).
__attribute__((visibility("default"))) int nd_set_pdl(int enable, int* previous) {
  if (previous != nullptr) *previous = nd::pdl_enabled() ? 1 : 0;
  nd::set_pdl_enabled(enable != 0);
  return ok();
}

__attribute__((visibility("default"))) int nd_set_sm_limit(int sms, int* previous) {
  if (sms < 0) return fail(ND_ERR_INVALID_ARG, "nd_set_sm_limit: sms = %d must be >= 0", sms);
  if (previous != nullptr) *previous = nd::sm_limit();
  nd::set_sm_limit(sms);
  return ok();
}

// Allocation-free variant of nd_kv_decode_attn for callers that may not call
// cudaMalloc: its scratch is the library's fixed 8 MiB per-GPU block
// (kv_decode_static_scratch), never a fresh allocation.  Same arguments and
// results as nd_kv_decode_attn minus the workspace.
__attribute__((visibility("default"))) int nd_kv_decode_attn_noalloc(
    void* stream, const void* q, const void* k_new, const void* v_new, void* k_cache,
    void* v_cache, void* out, int o_dtype, float* lse, int B, int H, int L, int L_max, int D,
    float scale) {
  if (B < 0 || H < 0) return fail(ND_ERR_INVALID_ARG, "nd_kv_decode_attn_noalloc: negative size");
  if (D != 64)
    return fail(ND_ERR_UNSUPPORTED, "nd_kv_decode_attn_noalloc: head_dim %d not supported (64 only)", D);
  if (L < 1 || L > L_max)
    return fail(ND_ERR_SHAPE, "nd_kv_decode_attn_noalloc: need 1 <= L <= L_max (L=%d, L_max=%d)", L, L_max);
  if (!valid_dtype(o_dtype))
    return fail(ND_ERR_UNSUPPORTED, "nd_kv_decode_attn_noalloc: bad o_dtype %d", o_dtype);
  if ((k_new == nullptr) != (v_new == nullptr))
    return fail(ND_ERR_INVALID_ARG,
                "nd_kv_decode_attn_noalloc: k_new and v_new must both be given or both NULL");
  if (static_cast<long long>(B) * H > 65535)
    return fail(ND_ERR_SHAPE, "nd_kv_decode_attn_noalloc: B*H = %lld exceeds 65535",
                static_cast<long long>(B) * H);
  if (B == 0 || H == 0) return ok();
  if (!q || !k_cache || !v_cache || !out)
    return fail(ND_ERR_INVALID_ARG, "nd_kv_decode_attn_noalloc: null tensor pointer");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out) ||
      (k_new && (!aligned16(k_new) || !aligned16(v_new))))
    return fail(ND_ERR_ALIGNMENT, "nd_kv_decode_attn_noalloc: tensors must be 16-byte aligned");
  const size_t need = nd::kv_decode_workspace_bytes(B, H, L);
  if (need > nd::kDecodeStaticScratchBytes)
    return fail(ND_ERR_WORKSPACE,
                "nd_kv_decode_attn_noalloc: B=%d H=%d L=%d needs %zu bytes of scratch, more than "
                "the %zu-byte fixed block of the allocation-free entry point; use "
                "nd_kv_decode_attn with a workspace",
                B, H, L, need, nd::kDecodeStaticScratchBytes);
  int dev = 0;
  int rc = check_current_device(&dev);
  if (rc) return rc;
  void* ws = nullptr;
  if (need > 0) {
    cudaError_t e = nd::kv_decode_static_scratch(dev, static_cast<cudaStream_t>(stream), &ws);
    if (e != cudaSuccess) return cuda_fail(e, "nd_kv_decode_attn_noalloc (scratch set-up)");
  }
  cudaError_t e = nd::launch_kv_decode(
      static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(q),
      static_cast<const __nv_bfloat16*>(k_new), static_cast<const __nv_bfloat16*>(v_new),
      static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), out,
      o_dtype == ND_F32, lse, B, H, L, L_max, scale, ws);
  if (e != cudaSuccess) return cuda_fail(e, "nd_kv_decode_attn_noalloc");
  return ok();
}

__attribute__((visibility("default"))) int nd_kv_append(void* stream, const void* k_new,
                                                        const void* v_new, void* k_cache,
                                                        void* v_cache, int B, int H, int pos,
                                                        int L_max, int D) {
  if (B < 0 || H < 0) return fail(ND_ERR_INVALID_ARG, "nd_kv_append: negative size");
  if (D <= 0 || D % 8) return fail(ND_ERR_UNSUPPORTED, "nd_kv_append: head_dim %d must be a positive multiple of 8", D);
  if (pos < 0 || pos >= L_max) return fail(ND_ERR_SHAPE, "nd_kv_append: pos %d outside [0, %d)", pos, L_max);
  if (B == 0 || H == 0) return ok();
  if (!k_new || !v_new || !k_cache || !v_cache) return fail(ND_ERR_INVALID_ARG, "nd_kv_append: null tensor pointer");
  if (!aligned16(k_new) || !aligned16(v_new) || !aligned16(k_cache) || !aligned16(v_cache))
    return fail(ND_ERR_ALIGNMENT, "nd_kv_append: tensors must be 16-byte aligned");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = nd::launch_kv_append(static_cast<cudaStream_t>(stream),
                                       static_cast<const __nv_bfloat16*>(k_new),
                                       static_cast<const __nv_bfloat16*>(v_new),
                                       static_cast<__nv_bfloat16*>(k_cache),
                                       static_cast<__nv_bfloat16*>(v_cache), B, H, pos, L_max, D);
  if (e != cudaSuccess) return cuda_fail(e, "nd_kv_append");
  return ok();
}

__attribute__((visibility("default"))) int nd_gemm_bias_act(void* stream, const void* A,
                                                            const void* W, const float* bias,
                                                            const void* residual,
                                                            int residual_dtype, void* Y,
                                                            int y_dtype, int M, int N, int K,
                                                            int act) {
  if (M < 0 || N < 0 || K < 0) return fail(ND_ERR_INVALID_ARG, "nd_gemm_bias_act: negative size");
  if (act < ND_ACT_NONE || act > ND_ACT_GELU_ERF) return fail(ND_ERR_UNSUPPORTED, "nd_gemm_bias_act: bad act %d", act);
  if (!valid_dtype(y_dtype) || (residual && !valid_dtype(residual_dtype)))
    return fail(ND_ERR_UNSUPPORTED, "nd_gemm_bias_act: bad dtype");
  if (M == 0 || N == 0) return ok();
  if (K == 0) return fail(ND_ERR_SHAPE, "nd_gemm_bias_act: K = 0");
  if (K % 8) return fail(ND_ERR_SHAPE, "nd_gemm_bias_act: K = %d must be a multiple of 8", K);
  if (!A || !W || !Y) return fail(ND_ERR_INVALID_ARG, "nd_gemm_bias_act: null tensor pointer");
  if (!aligned16(A) || !aligned16(W) || !aligned16(Y))
    return fail(ND_ERR_ALIGNMENT, "nd_gemm_bias_act: A/W/Y must be 16-byte aligned");
  if ((M + 127) / 128 > 65535) return fail(ND_ERR_SHAPE, "nd_gemm_bias_act: M too large");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  const char* msg = nullptr;
  cudaError_t e = nd::launch_gemm(static_cast<cudaStream_t>(stream),
                                  static_cast<const __nv_bfloat16*>(A),
                                  static_cast<const __nv_bfloat16*>(W), bias, residual,
                                  residual_dtype == ND_F32, Y, y_dtype == ND_F32, M, N, K, act, &msg);
  if (e != cudaSuccess) return cuda_fail(e, "nd_gemm_bias_act", msg);
  return ok();
}

// QKV projection of a prefill that also fills the decode caches.
__attribute__((visibility("default"))) int nd_gemm_qkv_cache(
    void* stream, const void* A, const void* W, const float* bias, void* Y, int M, int K,
    void* k_cache, void* v_cache, int B, int S, int H, int L_max, int pos0) {
  if (M < 0 || K < 0 || B < 0 || S < 0 || H < 0 || pos0 < 0)
    return fail(ND_ERR_INVALID_ARG, "nd_gemm_qkv_cache: negative size");
  if (static_cast<long long>(B) * S != M)
    return fail(ND_ERR_SHAPE, "nd_gemm_qkv_cache: M = %d rows but B*S = %lld", M,
                static_cast<long long>(B) * S);
  if (pos0 + S > L_max)
    return fail(ND_ERR_SHAPE, "nd_gemm_qkv_cache: positions [%d, %d) exceed L_max %d", pos0,
                pos0 + S, L_max);
  if (M == 0 || H == 0) return ok();
  if (K == 0 || K % 8) return fail(ND_ERR_SHAPE, "nd_gemm_qkv_cache: K = %d must be a positive multiple of 8", K);
  if (!A || !W || !Y || !k_cache || !v_cache)
    return fail(ND_ERR_INVALID_ARG, "nd_gemm_qkv_cache: null tensor pointer");
  if (!aligned16(A) || !aligned16(W) || !aligned16(Y) || !aligned16(k_cache) ||
      !aligned16(v_cache))
    return fail(ND_ERR_ALIGNMENT, "nd_gemm_qkv_cache: tensors must be 16-byte aligned");
  if (static_cast<long long>(B) * H > 65535)
    return fail(ND_ERR_SHAPE, "nd_gemm_qkv_cache: B*H exceeds 65535");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  const int dl = H * 64, N = 3 * dl;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const char* msg = nullptr;
  auto* kc = static_cast<__nv_bfloat16*>(k_cache);
  auto* vc = static_cast<__nv_bfloat16*>(v_cache);
  cudaError_t e;
  if (M > 32 && aligned16(bias)) {
    // the tensor-core path's bf16 staged epilogue writes the cache rows too
    nd::KvOut kv;
    kv.k = kc;
    kv.v = vc;
    kv.S = S;
    kv.H = H;
    kv.L_max = L_max;
    kv.pos0 = pos0;
    kv.dl = dl;
    e = nd::launch_gemm(st, static_cast<const __nv_bfloat16*>(A),
                        static_cast<const __nv_bfloat16*>(W), bias, nullptr, false, Y, false, M,
                        N, K, ND_ACT_NONE, &msg, kv);
  } else {
    // few rows (the weight-streaming path) or an unaligned bias: GEMM, then copy
    e = nd::launch_gemm(st, static_cast<const __nv_bfloat16*>(A),
                        static_cast<const __nv_bfloat16*>(W), bias, nullptr, false, Y, false, M,
                        N, K, ND_ACT_NONE, &msg);
    if (e == cudaSuccess)
      e = nd::launch_kv_store(st, static_cast<const __nv_bfloat16*>(Y), N, dl, 2 * dl, kc, vc, B,
                              S, H, L_max, pos0);
  }
  if (e != cudaSuccess) return cuda_fail(e, "nd_gemm_qkv_cache", msg);
  return ok();
}

// The QKV projection of a prompt-sharded prefill: the K/V columns of every
// head go straight to the cache of the rank that owns the head.
__attribute__((visibility("default"))) int nd_gemm_qkv_cache_peers(
    void* stream, const void* A, const void* W, const float* bias, void* Y, int M, int K,
    void* const* k_caches, void* const* v_caches, int tp, int B, int b0, int S, int H,
    int L_max, int pos0) {
  const char* fn = "nd_gemm_qkv_cache_peers";
  if (M < 0 || K < 0 || B < 0 || b0 < 0 || S < 0 || H < 0 || pos0 < 0)
    return fail(ND_ERR_INVALID_ARG, "%s: negative size", fn);
  if (tp < 1 || tp > nd::kKvMaxPeers) return fail(ND_ERR_INVALID_ARG, "%s: tp %d (1..%d)", fn, tp, nd::kKvMaxPeers);
  if (static_cast<long long>(B) * S != M)
    return fail(ND_ERR_SHAPE, "%s: M = %d rows but B*S = %lld", fn, M, static_cast<long long>(B) * S);
  if (pos0 + S > L_max)
    return fail(ND_ERR_SHAPE, "%s: positions [%d, %d) exceed L_max %d", fn, pos0, pos0 + S, L_max);
  if (M == 0 || H == 0) return ok();
  if (M <= 32) return fail(ND_ERR_UNSUPPORTED, "%s: %d rows (the cache-writing epilogue needs more than 32)", fn, M);
  if (K == 0 || K % 8) return fail(ND_ERR_SHAPE, "%s: K = %d must be a positive multiple of 8", fn, K);
  if (!A || !W || !Y || !k_caches || !v_caches) return fail(ND_ERR_INVALID_ARG, "%s: null pointer", fn);
  if (!aligned16(A) || !aligned16(W) || !aligned16(Y) || !aligned16(bias))
    return fail(ND_ERR_ALIGNMENT, "%s: A/W/Y/bias must be 16-byte aligned", fn);
  if (static_cast<long long>(b0 + B) * H > 65535) return fail(ND_ERR_SHAPE, "%s: (b0+B)*H exceeds 65535", fn);
  nd::KvOut kv;
  for (int q = 0; q < tp; ++q) {
    if (!k_caches[q] || !v_caches[q] || !aligned16(k_caches[q]) || !aligned16(v_caches[q]))
      return fail(ND_ERR_INVALID_ARG, "%s: cache of rank %d is NULL or unaligned", fn, q);
    kv.k_peer[q] = static_cast<__nv_bfloat16*>(k_caches[q]);
    kv.v_peer[q] = static_cast<__nv_bfloat16*>(v_caches[q]);
  }
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  const int dl = tp * H * 64, N = 3 * dl;
  kv.k = kv.k_peer[0];
  kv.v = kv.v_peer[0];
  kv.S = S;
  kv.H = H;
  kv.L_max = L_max;
  kv.pos0 = pos0;
  kv.dl = dl;
  kv.n_peers = tp;
  kv.b0 = b0;
  const char* msg = nullptr;
  cudaError_t e = nd::launch_gemm(static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(A),
                                  static_cast<const __nv_bfloat16*>(W), bias, nullptr, false, Y,
                                  false, M, N, K, ND_ACT_NONE, &msg, kv);
  if (e != cudaSuccess) return cuda_fail(e, fn, msg);
  return ok();
}

// Few-row linear layer with the residual add and LayerNorm in its prologue.
__attribute__((visibility("default"))) int nd_ln_gemm(void* stream, const void* x, const void* p,
                                                      const float* p_bias, const float* gamma,
                                                      const float* beta, float eps, void* s_out,
                                                      const void* W, const float* bias, void* Y,
                                                      int y_dtype, int M, int N, int K, int act) {
  if (M < 0 || N < 0 || K < 0) return fail(ND_ERR_INVALID_ARG, "nd_ln_gemm: negative size");
  if (act < ND_ACT_NONE || act > ND_ACT_GELU_ERF)
    return fail(ND_ERR_UNSUPPORTED, "nd_ln_gemm: bad act %d", act);
  if (!valid_dtype(y_dtype)) return fail(ND_ERR_UNSUPPORTED, "nd_ln_gemm: bad y dtype %d", y_dtype);
  if (M > nd::kLnGemmMaxRows)
    return fail(ND_ERR_SHAPE, "nd_ln_gemm: M = %d rows, at most %d", M, nd::kLnGemmMaxRows);
  if (K == 0 || K % 32 != 0 || K > nd::kLnGemmMaxK)
    return fail(ND_ERR_SHAPE, "nd_ln_gemm: K = %d must be a multiple of 32 in [32, %d]", K,
                nd::kLnGemmMaxK);
  if (M == 0 || N == 0) return ok();
  if (!x || !W || !Y) return fail(ND_ERR_INVALID_ARG, "nd_ln_gemm: null tensor pointer");
  if (!aligned16(x) || !aligned16(W) || !aligned16(Y) || (p && !aligned16(p)) ||
      (s_out && !aligned16(s_out)) || (p_bias && !aligned16(p_bias)) ||
      (gamma && !aligned16(gamma)) || (beta && !aligned16(beta)))
    return fail(ND_ERR_ALIGNMENT, "nd_ln_gemm: tensors and parameter vectors must be 16-byte aligned");
  if (s_out) {
    // every CTA reads x and p while CTA 0 writes s_out
    const size_t bytes = static_cast<size_t>(M) * K * 2;
    auto overlaps = [&](const void* a) {
      const uintptr_t u = reinterpret_cast<uintptr_t>(a), v = reinterpret_cast<uintptr_t>(s_out);
      return a != nullptr && u < v + bytes && v < u + bytes;
    };
    if (overlaps(x) || overlaps(p))
      return fail(ND_ERR_INVALID_ARG, "nd_ln_gemm: s_out must not overlap x or p");
  }
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = nd::launch_ln_gemm(
      static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x),
      static_cast<const __nv_bfloat16*>(p), p_bias, gamma, beta, eps,
      static_cast<__nv_bfloat16*>(s_out), static_cast<const __nv_bfloat16*>(W), bias, Y,
      y_dtype == ND_F32, M, N, K, act);
  if (e != cudaSuccess) return cuda_fail(e, "nd_ln_gemm");
  return ok();
}

// Unfused graph ops (fp32): :gelu, :scale_mask (causal), :softmax.
__attribute__((visibility("default"))) int nd_gelu(void* stream, const float* x, float* y,
                                                   int64_t n, int act) {
  if (n < 0) return fail(ND_ERR_INVALID_ARG, "nd_gelu: negative size");
  if (act < ND_ACT_GELU_SIGMOID || act > ND_ACT_GELU_ERF)
    return fail(ND_ERR_UNSUPPORTED, "nd_gelu: act %d is not a GELU form", act);
  if (n == 0) return ok();
  if (!x || !y) return fail(ND_ERR_INVALID_ARG, "nd_gelu: null pointer");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = nd::launch_gelu(static_cast<cudaStream_t>(stream), x, y, n, act);
  if (e != cudaSuccess) return cuda_fail(e, "nd_gelu");
  return ok();
}

__attribute__((visibility("default"))) int nd_scale_mask(void* stream, const float* x, float* y,
                                                         int rows, int cols, int d_head) {
  if (rows < 0 || cols < 0) return fail(ND_ERR_INVALID_ARG, "nd_scale_mask: negative size");
  if (d_head <= 0) return fail(ND_ERR_INVALID_ARG, "nd_scale_mask: d_head = %d", d_head);
  if (static_cast<long long>(rows) * cols == 0) return ok();
  if (!x || !y) return fail(ND_ERR_INVALID_ARG, "nd_scale_mask: null pointer");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = nd::launch_scale_mask(static_cast<cudaStream_t>(stream), x, y, rows, cols,
                                        1.f / sqrtf(static_cast<float>(d_head)));
  if (e != cudaSuccess) return cuda_fail(e, "nd_scale_mask");
  return ok();
}

__attribute__((visibility("default"))) int nd_add(void* stream, const float* a, const float* b,
                                                  float* y, int rows, int cols, int b_mode) {
  if (rows < 0 || cols < 0) return fail(ND_ERR_INVALID_ARG, "nd_add: negative size");
  if (b_mode < 0 || b_mode > 3) return fail(ND_ERR_INVALID_ARG, "nd_add: b_mode %d", b_mode);
  if (static_cast<long long>(rows) * cols == 0) return ok();
  if (!a || !b || !y) return fail(ND_ERR_INVALID_ARG, "nd_add: null pointer");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = nd::launch_add(static_cast<cudaStream_t>(stream), a, b, y, rows, cols, b_mode);
  if (e != cudaSuccess) return cuda_fail(e, "nd_add");
  return ok();
}

__attribute__((visibility("default"))) int nd_softmax(void* stream, const float* x, float* y,
                                                      int rows, int cols) {
  if (rows < 0 || cols < 0) return fail(ND_ERR_INVALID_ARG, "nd_softmax: negative size");
  if (static_cast<long long>(rows) * cols == 0) return ok();
  if (!x || !y) return fail(ND_ERR_INVALID_ARG, "nd_softmax: null pointer");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = nd::launch_softmax(static_cast<cudaStream_t>(stream), x, y, rows, cols);
  if (e != cudaSuccess) return cuda_fail(e, "nd_softmax");
  return ok();
}

__attribute__((visibility("default"))) int nd_layernorm(void* stream, const void* x, int x_dtype,
                                                        const float* gamma, const float* beta,
                                                        void* y, int y_dtype, float* mean,
                                                        float* rstd, int rows, int d, float eps) {
  if (rows < 0 || d < 0) return fail(ND_ERR_INVALID_ARG, "nd_layernorm: negative size");
  if (!valid_dtype(x_dtype) || !valid_dtype(y_dtype)) return fail(ND_ERR_UNSUPPORTED, "nd_layernorm: bad dtype");
  if (rows == 0) return ok();
  if (d == 0) return fail(ND_ERR_SHAPE, "nd_layernorm: d = 0");
  if (!x || !y) return fail(ND_ERR_INVALID_ARG, "nd_layernorm: null tensor pointer");
  if (static_cast<size_t>(d) * sizeof(float) > 200 * 1024)
    return fail(ND_ERR_SHAPE, "nd_layernorm: d = %d too large", d);
  if (rows > 0x7fffffff / 8) return fail(ND_ERR_SHAPE, "nd_layernorm: too many rows");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  const bool vec_ok = (d % 8 == 0) && aligned16(x) && aligned16(y) &&
                      (!gamma || aligned16(gamma)) && (!beta || aligned16(beta));
  cudaError_t e = nd::launch_layernorm(static_cast<cudaStream_t>(stream), x, x_dtype == ND_BF16,
                                       gamma, beta, y, y_dtype == ND_BF16, mean, rstd, rows, d, eps,
                                       vec_ok);
  if (e != cudaSuccess) return cuda_fail(e, "nd_layernorm");
  return ok();
}

static int convert_2d_impl(const char* fn, void* stream, const void* src, int src_dtype,
                           int src_col_major, void* dst, int dst_dtype, int rows, int cols,
                           int ld_dst) {
  if (rows < 0 || cols < 0) return fail(ND_ERR_INVALID_ARG, "%s: negative size", fn);
  if (ld_dst < cols) return fail(ND_ERR_SHAPE, "%s: ld_dst %d < cols %d", fn, ld_dst, cols);
  if (!valid_dtype(src_dtype) || !valid_dtype(dst_dtype)) return fail(ND_ERR_UNSUPPORTED, "%s: bad dtype", fn);
  if (rows == 0 || ld_dst == 0) return ok();
  if (!dst || (cols > 0 && !src)) return fail(ND_ERR_INVALID_ARG, "%s: null pointer", fn);
  if ((rows + 31) / 32 > 65535) return fail(ND_ERR_SHAPE, "%s: too many rows", fn);
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool cm = src_col_major != 0;
  cudaError_t e;
  if (src_dtype == ND_F32 && dst_dtype == ND_F32) e = launch_convert<float, float>(st, src, dst, rows, cols, cm, ld_dst);
  else if (src_dtype == ND_F32) e = launch_convert<float, __nv_bfloat16>(st, src, dst, rows, cols, cm, ld_dst);
  else if (dst_dtype == ND_F32) e = launch_convert<__nv_bfloat16, float>(st, src, dst, rows, cols, cm, ld_dst);
  else e = launch_convert<__nv_bfloat16, __nv_bfloat16>(st, src, dst, rows, cols, cm, ld_dst);
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return ok();
}

__attribute__((visibility("default"))) int nd_convert_2d(void* stream, const void* src,
                                                         int src_dtype, int src_col_major,
                                                         void* dst, int dst_dtype, int rows,
                                                         int cols) {
  return convert_2d_impl("nd_convert_2d", stream, src, src_dtype, src_col_major, dst, dst_dtype,
                         rows, cols, cols);
}

__attribute__((visibility("default"))) int nd_convert_2d_padded(void* stream, const void* src,
                                                                int src_dtype, int src_col_major,
                                                                void* dst, int dst_dtype, int rows,
                                                                int cols, int ld_dst) {
  return convert_2d_impl("nd_convert_2d_padded", stream, src, src_dtype, src_col_major, dst,
                         dst_dtype, rows, cols, ld_dst);
}

__attribute__((visibility("default"))) int nd_gather_rows(void* stream, const void* table,
                                                          int dtype, long long ld_table, int vocab,
                                                          const void* idx, int idx_dtype,
                                                          int index_base, int n, int d, void* out,
                                                          long long ld_out) {
  if (n < 0 || d < 0 || vocab < 0) return fail(ND_ERR_INVALID_ARG, "nd_gather_rows: negative size");
  if (!valid_dtype(dtype)) return fail(ND_ERR_UNSUPPORTED, "nd_gather_rows: bad dtype %d", dtype);
  if (idx_dtype != ND_F32 && idx_dtype != ND_I32 && idx_dtype != ND_I64)
    return fail(ND_ERR_UNSUPPORTED, "nd_gather_rows: bad index dtype %d", idx_dtype);
  if (ld_table < d || ld_out < d)
    return fail(ND_ERR_SHAPE, "nd_gather_rows: row strides (%lld, %lld) below d = %d", ld_table,
                ld_out, d);
  if (n == 0 || d == 0) return ok();
  if (!table || !idx || !out) return fail(ND_ERR_INVALID_ARG, "nd_gather_rows: null pointer");
  if (vocab == 0) return fail(ND_ERR_SHAPE, "nd_gather_rows: empty table");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = nd::launch_gather_rows(static_cast<cudaStream_t>(stream), table,
                                         dtype == ND_F32 ? 4 : 2, ld_table, vocab, idx,
                                         idx_dtype == ND_F32 ? 0 : idx_dtype == ND_I32 ? 1 : 2,
                                         index_base, n, d, out, ld_out, nd::device_error_word());
  if (e != cudaSuccess) return cuda_fail(e, "nd_gather_rows");
  return ok();
}

__attribute__((visibility("default"))) int nd_copy_2d(void* stream, const void* src,
                                                      long long ld_src, void* dst,
                                                      long long ld_dst, int rows, int cols,
                                                      int elem_bytes) {
  if (rows < 0 || cols < 0) return fail(ND_ERR_INVALID_ARG, "nd_copy_2d: negative size");
  if (elem_bytes != 2 && elem_bytes != 4)
    return fail(ND_ERR_UNSUPPORTED, "nd_copy_2d: element size %d (2 or 4)", elem_bytes);
  if (ld_src < cols || ld_dst < cols)
    return fail(ND_ERR_SHAPE, "nd_copy_2d: row strides (%lld, %lld) below cols = %d", ld_src,
                ld_dst, cols);
  if (rows == 0 || cols == 0) return ok();
  if (!src || !dst) return fail(ND_ERR_INVALID_ARG, "nd_copy_2d: null pointer");
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) % elem_bytes)
    return fail(ND_ERR_ALIGNMENT, "nd_copy_2d: pointers not aligned to the element size");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = nd::launch_copy_2d(static_cast<cudaStream_t>(stream), src, ld_src, dst, ld_dst,
                                     rows, cols, elem_bytes);
  if (e != cudaSuccess) return cuda_fail(e, "nd_copy_2d");
  return ok();
}

__attribute__((visibility("default"))) int nd_copy_2d_batched(
    void* stream, const void* src, long long ld_src, long long bs_src, void* dst, long long ld_dst,
    long long bs_dst, int batch, int rows, int cols, int elem_bytes) {
  const char* fn = "nd_copy_2d_batched";
  if (rows < 0 || cols < 0 || batch < 0) return fail(ND_ERR_INVALID_ARG, "%s: negative size", fn);
  if (batch > 65535) return fail(ND_ERR_SHAPE, "%s: batch %d above 65535", fn, batch);
  if (elem_bytes != 2 && elem_bytes != 4)
    return fail(ND_ERR_UNSUPPORTED, "%s: element size %d (2 or 4)", fn, elem_bytes);
  if (ld_src < cols || ld_dst < cols)
    return fail(ND_ERR_SHAPE, "%s: row strides (%lld, %lld) below cols = %d", fn, ld_src, ld_dst, cols);
  if (batch > 1 && (bs_src < 0 || bs_dst < 0))
    return fail(ND_ERR_SHAPE, "%s: negative batch stride", fn);
  if (rows == 0 || cols == 0 || batch == 0) return ok();
  if (!src || !dst) return fail(ND_ERR_INVALID_ARG, "%s: null pointer", fn);
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) % elem_bytes)
    return fail(ND_ERR_ALIGNMENT, "%s: pointers not aligned to the element size", fn);
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = nd::launch_copy_2d(static_cast<cudaStream_t>(stream), src, ld_src, dst, ld_dst,
                                     rows, cols, elem_bytes, batch, bs_src, bs_dst);
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return ok();
}

__attribute__((visibility("default"))) int nd_embed(void* stream, const int32_t* ids,
                                                    const int32_t* pos, const void* wte,
                                                    const void* wpe, void* y, int T, int d,
                                                    int vocab, int n_pos) {
  if (T < 0 || d < 0 || vocab < 0 || n_pos < 0) return fail(ND_ERR_INVALID_ARG, "nd_embed: negative size");
  if (d % 8 != 0) return fail(ND_ERR_SHAPE, "nd_embed: d = %d must be a multiple of 8", d);
  if (T == 0 || d == 0) return ok();
  if (!ids || !wte || !y || (pos && !wpe)) return fail(ND_ERR_INVALID_ARG, "nd_embed: null pointer");
  if (!aligned16(wte) || !aligned16(y) || (wpe && !aligned16(wpe)))
    return fail(ND_ERR_ALIGNMENT, "nd_embed: wte/wpe/y must be 16-byte aligned");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = nd::launch_embed(static_cast<cudaStream_t>(stream), ids, pos,
                                   static_cast<const __nv_bfloat16*>(wte),
                                   static_cast<const __nv_bfloat16*>(wpe),
                                   static_cast<__nv_bfloat16*>(y), T, d, vocab, n_pos,
                                   nd::device_error_word());
  if (e != cudaSuccess) return cuda_fail(e, "nd_embed");
  return ok();
}

__attribute__((visibility("default"))) int nd_argmax(void* stream, const void* logits, int dtype,
                                                     int64_t ld, int rows, int V, int32_t* idx,
                                                     float* val) {
  if (rows < 0 || V < 0) return fail(ND_ERR_INVALID_ARG, "nd_argmax: negative size");
  if (!valid_dtype(dtype)) return fail(ND_ERR_UNSUPPORTED, "nd_argmax: bad dtype %d", dtype);
  if (ld < V) return fail(ND_ERR_SHAPE, "nd_argmax: ld %lld < V %d", static_cast<long long>(ld), V);
  if (rows == 0) return ok();
  if (V == 0) return fail(ND_ERR_SHAPE, "nd_argmax: empty rows (V = 0)");
  if (!logits || !idx) return fail(ND_ERR_INVALID_ARG, "nd_argmax: null pointer");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = nd::launch_argmax(static_cast<cudaStream_t>(stream), logits, dtype == ND_F32, ld,
                                    rows, V, idx, val);
  if (e != cudaSuccess) return cuda_fail(e, "nd_argmax");
  return ok();
}

__attribute__((visibility("default"))) int nd_kv_store(void* stream, const void* src, int64_t ld,
                                                       int k_col, int v_col, void* k_cache,
                                                       void* v_cache, int B, int S, int H,
                                                       int L_max, int pos0, int D) {
  if (B < 0 || S < 0 || H < 0 || L_max < 0 || pos0 < 0) return fail(ND_ERR_INVALID_ARG, "nd_kv_store: negative size");
  if (D != 64) return fail(ND_ERR_UNSUPPORTED, "nd_kv_store: head_dim %d not supported (64 only)", D);
  if (pos0 + static_cast<long long>(S) > L_max)
    return fail(ND_ERR_SHAPE, "nd_kv_store: pos0 %d + S %d exceeds L_max %d", pos0, S, L_max);
  if (ld % 8 || k_col % 8 || v_col % 8 || k_col < 0 || v_col < 0 ||
      k_col + static_cast<long long>(H) * 64 > ld || v_col + static_cast<long long>(H) * 64 > ld)
    return fail(ND_ERR_SHAPE, "nd_kv_store: columns k=%d v=%d (+%d) must be multiples of 8 inside ld=%lld",
                k_col, v_col, H * 64, static_cast<long long>(ld));
  if (B == 0 || S == 0 || H == 0) return ok();
  if (!src || !k_cache || !v_cache) return fail(ND_ERR_INVALID_ARG, "nd_kv_store: null pointer");
  if (!aligned16(src) || !aligned16(k_cache) || !aligned16(v_cache))
    return fail(ND_ERR_ALIGNMENT, "nd_kv_store: tensors must be 16-byte aligned");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = nd::launch_kv_store(static_cast<cudaStream_t>(stream),
                                      static_cast<const __nv_bfloat16*>(src), ld, k_col, v_col,
                                      static_cast<__nv_bfloat16*>(k_cache),
                                      static_cast<__nv_bfloat16*>(v_cache), B, S, H, L_max, pos0);
  if (e != cudaSuccess) return cuda_fail(e, "nd_kv_store");
  return ok();
}

__attribute__((visibility("default"))) int nd_add_layernorm(void* stream, const void* x,
                                                            const void* p, int p_dtype,
                                                            const float* bias, const float* gamma,
                                                            const float* beta, void* s_out,
                                                            void* y, int rows, int d, float eps) {
  if (rows < 0 || d < 0) return fail(ND_ERR_INVALID_ARG, "nd_add_layernorm: negative size");
  if (!valid_dtype(p_dtype)) return fail(ND_ERR_UNSUPPORTED, "nd_add_layernorm: bad p dtype %d", p_dtype);
  if (d % 8 != 0 || d > 2048 || d == 0)
    return fail(ND_ERR_SHAPE, "nd_add_layernorm: d = %d must be a multiple of 8 in [8, 2048]", d);
  if (rows == 0) return ok();
  if (!x || !p || !s_out || !y) return fail(ND_ERR_INVALID_ARG, "nd_add_layernorm: null pointer");
  if (!aligned16(x) || !aligned16(p) || !aligned16(s_out) || !aligned16(y))
    return fail(ND_ERR_ALIGNMENT, "nd_add_layernorm: tensors must be 16-byte aligned");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaError_t e = nd::launch_add_layernorm(
      static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x), p, p_dtype == ND_F32,
      bias, gamma, beta, static_cast<__nv_bfloat16*>(s_out), static_cast<__nv_bfloat16*>(y), rows, d,
      eps);
  if (e != cudaSuccess) return cuda_fail(e, "nd_add_layernorm");
  return ok();
}

__attribute__((visibility("default"))) int nd_comm_region_bytes(int rows_max, int d,
                                                                size_t* bytes) {
  if (!bytes) return fail(ND_ERR_INVALID_ARG, "nd_comm_region_bytes: bytes is NULL");
  if (rows_max < 1 || d < 8 || d % 8 || d > 2048)
    return fail(ND_ERR_SHAPE, "nd_comm_region_bytes: rows_max %d, d %d (d a multiple of 8 in [8, 2048])",
                rows_max, d);
  *bytes = nd::comm_region_bytes(rows_max, d);
  return ok();
}

__attribute__((visibility("default"))) int nd_comm_slot_offset(int slot, int rows_max, int d,
                                                               size_t* offset) {
  if (!offset) return fail(ND_ERR_INVALID_ARG, "nd_comm_slot_offset: offset is NULL");
  if ((slot != 0 && slot != 1) || rows_max < 1 || d < 8 || d % 8 || d > 2048)
    return fail(ND_ERR_SHAPE, "nd_comm_slot_offset: slot %d, rows_max %d, d %d", slot, rows_max, d);
  *offset = nd::comm_slot_offset(slot, rows_max, d);
  return ok();
}

__attribute__((visibility("default"))) int nd_comm_alloc(size_t bytes, void** region,
                                                         void* ipc_handle) {
  if (!region || !ipc_handle) return fail(ND_ERR_INVALID_ARG, "nd_comm_alloc: null pointer");
  if (bytes < nd::comm_region_bytes(1, 8)) return fail(ND_ERR_SHAPE, "nd_comm_alloc: %zu bytes is too small", bytes);
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "nd_comm_alloc: cudaMalloc");
  // flags and sequence counters start at zero; finished before any peer sees the handle
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "nd_comm_alloc");
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *region = p;
  return ok();
}

__attribute__((visibility("default"))) int nd_comm_open(const void* ipc_handle, void** peer_region) {
  if (!ipc_handle || !peer_region) return fail(ND_ERR_INVALID_ARG, "nd_comm_open: null pointer");
  int rc = check_current_device(nullptr);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "nd_comm_open: cudaIpcOpenMemHandle");
  *peer_region = p;
  return ok();
}

__attribute__((visibility("default"))) int nd_comm_close(void* peer_region) {
  if (!peer_region) return ok();
  cudaError_t e = cudaIpcCloseMemHandle(peer_region);
  if (e != cudaSuccess) return cuda_fail(e, "nd_comm_close");
  return ok();
}

__attribute__((visibility("default"))) int nd_comm_free(void* region) {
  if (!region) return ok();
  cudaError_t e = cudaFree(region);
  if (e != cudaSuccess) return cuda_fail(e, "nd_comm_free");
  return ok();
}

__attribute__((visibility("default"))) int nd_allreduce_add_layernorm(
    void* stream, void* const* regions, int tp, int rank, size_t region_bytes, int rows_max,
    int slot, const void* x, const float* bias, const float* gamma, const float* beta,
    void* s_out, void* y, int rows, int d, float eps) {
  if (!regions) return fail(ND_ERR_INVALID_ARG, "nd_allreduce_add_layernorm: regions is NULL");
  if (tp < 1 || tp > nd::kCommMaxRanks || rank < 0 || rank >= tp)
    return fail(ND_ERR_INVALID_ARG, "nd_allreduce_add_layernorm: tp %d / rank %d (tp <= %d)", tp, rank,
                nd::kCommMaxRanks);
  if (slot != 0 && slot != 1) return fail(ND_ERR_INVALID_ARG, "nd_allreduce_add_layernorm: slot %d (0 or 1)", slot);
  if (d < 8 || d % 8 || d > 2048)
    return fail(ND_ERR_SHAPE, "nd_allreduce_add_layernorm: d = %d must be a multiple of 8 in [8, 2048]", d);
  if (rows < 0 || rows > rows_max)
    return fail(ND_ERR_SHAPE, "nd_allreduce_add_layernorm: rows %d outside [0, rows_max %d]", rows, rows_max);
  if (nd::comm_region_bytes(rows_max, d) > region_bytes)
    return fail(ND_ERR_SHAPE, "nd_allreduce_add_layernorm: %zu-byte regions cannot hold %d x %d slots",
                region_bytes, rows_max, d);
  if (rows == 0) return ok();
  if (!x || !s_out || !y) return fail(ND_ERR_INVALID_ARG, "nd_allreduce_add_layernorm: null tensor pointer");
  if (!aligned16(x) || !aligned16(s_out) || !aligned16(y))
    return fail(ND_ERR_ALIGNMENT, "nd_allreduce_add_layernorm: x/s_out/y must be 16-byte aligned");
  nd::CommRegions regs = {};
  for (int r = 0; r < tp; ++r) {
    if (!regions[r] || !aligned16(regions[r]))
      return fail(ND_ERR_INVALID_ARG, "nd_allreduce_add_layernorm: region %d is NULL or unaligned", r);
    regs.r[r] = regions[r];
  }
  int dev = 0;
  int rc = check_current_device(&dev);
  if (rc) return rc;
  int sms = 0;
  cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess)
    e = nd::launch_allreduce_add_layernorm(
        static_cast<cudaStream_t>(stream), regs, tp, rank, slot, rows_max,
        static_cast<const __nv_bfloat16*>(x), bias, gamma, beta,
        static_cast<__nv_bfloat16*>(s_out), static_cast<__nv_bfloat16*>(y), rows, d, eps, sms,
        nd::device_error_word());
  if (e != cudaSuccess) return cuda_fail(e, "nd_allreduce_add_layernorm");
  return ok();
}

__attribute__((visibility("default"))) int nd_gemm_allreduce_add_layernorm(
    void* stream, const void* A, const void* W, int K, void* const* regions, int tp, int rank,
    size_t region_bytes, int rows_max, int slot, const void* x, const float* bias,
    const float* gamma, const float* beta, void* s_out, void* y, int rows, int d, float eps) {
  const char* fn = "nd_gemm_allreduce_add_layernorm";
  if (!regions) return fail(ND_ERR_INVALID_ARG, "%s: regions is NULL", fn);
  if (tp < 1 || tp > nd::kCommMaxRanks || rank < 0 || rank >= tp)
    return fail(ND_ERR_INVALID_ARG, "%s: tp %d / rank %d (tp <= %d)", fn, tp, rank, nd::kCommMaxRanks);
  if (slot != 0 && slot != 1) return fail(ND_ERR_INVALID_ARG, "%s: slot %d (0 or 1)", fn, slot);
  if (rows < 0 || rows > rows_max)
    return fail(ND_ERR_SHAPE, "%s: rows %d outside [0, rows_max %d]", fn, rows, rows_max);
  if (rows == 0) return ok();
  if (!nd::fused_projection_supported(tp, rows, d, K))
    return fail(ND_ERR_UNSUPPORTED,
                "%s: tp %d rows %d d %d K %d (tp 1, 2, 4 or 8; rows <= 32; d a multiple of 8 up to 1024; "
                "K a multiple of 32)", fn, tp, rows, d, K);
  if (nd::comm_region_bytes(rows_max, d) > region_bytes)
    return fail(ND_ERR_SHAPE, "%s: %zu-byte regions cannot hold %d x %d slots", fn, region_bytes,
                rows_max, d);
  if (!A || !W || !x || !s_out || !y) return fail(ND_ERR_INVALID_ARG, "%s: null tensor pointer", fn);
  if (!aligned16(A) || !aligned16(W) || !aligned16(x) || !aligned16(s_out) || !aligned16(y))
    return fail(ND_ERR_ALIGNMENT, "%s: A/W/x/s_out/y must be 16-byte aligned", fn);
  nd::CommRegions regs = {};
  for (int r = 0; r < tp; ++r) {
    if (!regions[r] || !aligned16(regions[r]))
      return fail(ND_ERR_INVALID_ARG, "%s: region %d is NULL or unaligned", fn, r);
    regs.r[r] = regions[r];
  }
  int dev = 0;
  int rc = check_current_device(&dev);
  if (rc) return rc;
  cudaError_t e = nd::launch_gemm_allreduce_add_layernorm(
      static_cast<cudaStream_t>(stream), regs, tp, rank, slot, rows_max,
      static_cast<const __nv_bfloat16*>(A), static_cast<const __nv_bfloat16*>(W), K,
      static_cast<const __nv_bfloat16*>(x), bias, gamma, beta,
      static_cast<__nv_bfloat16*>(s_out), static_cast<__nv_bfloat16*>(y), rows, d, eps,
      nd::device_error_word());
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return ok();
}

}  // extern "C"
