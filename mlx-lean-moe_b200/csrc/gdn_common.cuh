// Shared device helpers and the internal launch interface of libgdn_b200.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <utility>

#include "gdn_api.h"

namespace gdn {

// ---------------------------------------------------------------------------
// Per-device one-time set-up.  Function attributes (the opt-in to more than
// 48 KB of dynamic shared memory) belong to each device's context, so one
// process driving several GPUs must set them on every device it launches on.
// The flags are atomics: host threads may launch concurrently; a repeat of
// cudaFuncSetAttribute from a racing thread is harmless.
// ---------------------------------------------------------------------------
constexpr int kMaxDevices = 64;
struct DeviceFlags {
  std::atomic<bool> set[kMaxDevices];
};

template <typename K>
cudaError_t ensure_smem_attr(K* kernel, size_t bytes, DeviceFlags& flags) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const bool cached = dev >= 0 && dev < kMaxDevices;
  if (cached && flags.set[dev].load(std::memory_order_acquire)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess && cached) flags.set[dev].store(true, std::memory_order_release);
  return e;
}

// The current device's SM count, looked up once per device (148 when the
// lookup fails, which only sizes grids).
inline int sm_count() {
  static std::atomic<int> cached[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  const bool in_range = dev >= 0 && dev < kMaxDevices;
  if (in_range) {
    const int c = cached[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  if (in_range) cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

// ---------------------------------------------------------------------------
// Element loads/stores with conversion to/from float
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// Round a float to the precision of T and back (identity for float).
template <typename T>
__device__ __forceinline__ float round_to(float x) { return to_f(from_f<T>(x)); }

// Two floats to bf16 (round to nearest even) in one packed conversion: on
// sm_100 it has about four times the per-value throughput of the scalar
// conversion, which shares the special-function pipe with exp2 / rcp.
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void round2_bf16(float& a, float& b) {
  const uint32_t w = cvt_bf16x2(a, b);
  a = __uint_as_float(w << 16);
  b = __uint_as_float(w & 0xFFFF0000u);
}
// Round 8 floats to the precision of T (pairwise for bf16).
template <typename T>
__device__ __forceinline__ void round8(float (&x)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = round_to<T>(x[i]);
}
template <>
__device__ __forceinline__ void round8<float>(float (&)[8]) {}
template <>
__device__ __forceinline__ void round8<__nv_bfloat16>(float (&x)[8]) {
#pragma unroll
  for (int i = 0; i < 8; i += 2) round2_bf16(x[i], x[i + 1]);
}

// Packed fp32 pair arithmetic (sm_100 f32x2): two independent IEEE fp32
// operations with round-to-nearest per instruction, bit-identical to the
// scalar fmaf / fmul pairs they replace.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float4 operator*(float4 a, float s) { return make_float4(a.x * s, a.y * s, a.z * s, a.w * s); }
__device__ __forceinline__ float dot4(float4 a, float4 b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }

// Token range of sequence b.
__device__ __forceinline__ void seq_range(const int64_t* cu, int64_t n_tokens, int64_t n_seqs, int64_t b,
                                          int64_t& start, int64_t& end) {
  if (cu) {
    start = cu[b];
    end = cu[b + 1];
  } else {
    const int64_t len = n_tokens / n_seqs;
    start = b * len;
    end = start + len;
  }
}

// softplus(x) = log(1 + exp(x)) without overflow.
__device__ __forceinline__ float softplus_f(float x) { return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x))); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return x / (1.f + expf(-x)); }
// x * sigmoid(x) as x / (1 + 2^(-x log2 e)) with the hardware approximate
// exp2 (ex2.approx) and the approximate divide: a few instructions, relative error ~1e-6 (well below the bf16
// rounding that follows it in the fused-block kernels).  For x < -87 the
// denominator is inf and the result the correct limit -0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.f + ex2_approx(x * -1.4426950408889634f)); }

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched by launch_dependent() may
// start while the kernel before it on the stream is still running;
// griddep_wait() blocks until that kernel has completed and its memory writes
// are visible (at once when there is no such kernel or the launch was a
// plain one).  Every kernel launched by launch_dependent() calls
// griddep_wait() in every CTA before it reads or writes memory that earlier
// work may touch, so completion stays ordered along the stream.
// griddep_launch_dependents() lets the next dependent launch begin.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                             Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// Internal launch interface (one struct, filled by gdn_api.cu after checks)
// ---------------------------------------------------------------------------
struct ScanParams {
  int64_t n_tokens, n_seqs;
  const int64_t* cu_seqlens;
  int hk, hv, dk, dv;
  const void *q, *k, *v, *g, *beta;
  int64_t q_st, q_sh, k_st, k_sh, v_st, v_sh, g_st, beta_st;
  const float* state_in;
  float* state_out;
  void* out;
  gdn_dtype qkv_dtype, gate_dtype, out_dtype;
  gdn_gate_kind gate_kind;
  // decode only
  const int32_t* state_slots;
  // chunked only
  void* workspace;
  size_t workspace_bytes;
  // chunked, optional (z != nullptr): out = silu(z) * rms_norm(y -> out dtype,
  // norm_w, eps) in the output stage (the fused block's gated norm); z is
  // [N, Hv, Dv] in the out dtype with token stride z_st and head stride Dv.
  const void* z = nullptr;
  int64_t z_st = 0;
  const float* norm_w = nullptr;
  float norm_eps = 0.f;
  // chunked, optional: `out` is a [N, out_hv, Dv] gathered output holding
  // this call's heads at [head0, head0 + hv); every output tile is also
  // written to the n_peers other ranks' gathered outputs (gdn_scan_gathered).
  int out_hv = 0;  // 0: hv
  int head0 = 0;
  int n_peers = 0;
  void* peer_out[GDN_MAX_GATHER_PEERS] = {};
};

struct BlockParams {
  int64_t n_tokens, n_seqs;
  const int64_t* cu_seqlens;
  int hk, hv, dk, dv, kernel;
  const void* mixed;
  int64_t mixed_st;
  gdn_dtype act_dtype;
  const float* conv_w;
  const void* conv_state_in;
  void* conv_state_out;
  gdn_dtype conv_state_dtype;
  const float *A_log, *dt_bias, *norm_w;
  float eps;
  // prologue outputs (workspace)
  void *q, *k, *v;   // act dtype, [N, Hk, Dk], [N, Hk, Dk], [N, Hv, Dv]
  float *g_log, *beta;  // [N, Hv]
  void* y;           // [N, Hv, Dv] scan output in the act dtype (the reference
                     // casts y to it before the gated norm)
  void* out;         // [N, Hv, Dv] act dtype
};

// Records a printf-style message for gdn_last_error() and returns st.
gdn_status set_error(gdn_status st, const char* fmt, ...);
gdn_status allocation_range(const void* ptr, void** base, size_t* size);

cudaError_t launch_decode(const ScanParams& p, cudaStream_t s);
cudaError_t launch_serial_scan(const ScanParams& p, cudaStream_t s);
bool serial_supported(int dk);

cudaError_t launch_forget_gate(const void* a, gdn_dtype dt, int64_t a_st, int64_t n, int hv, const float* A_log,
                               const float* dt_bias, float* g, gdn_gate_kind kind, cudaStream_t s);

cudaError_t launch_block_prologue(const BlockParams& p, cudaStream_t s);
cudaError_t launch_block_conv_tail(const BlockParams& p, cudaStream_t s);
cudaError_t launch_block_epilogue(const BlockParams& p, cudaStream_t s);
// Every sequence one token, Dk = Dv = 128, conv width <= 4, the conv tail
// written apart from the conv state it reads: the whole block in one kernel.
bool block_decode_supported(const BlockParams& p, const float* state_in, const float* state_out);
cudaError_t launch_block_decode(const BlockParams& p, const float* state_in, float* state_out, cudaStream_t s);

// Chunked (tensor-core) prefill.
bool chunked_supported(const ScanParams& p);
size_t chunked_workspace_bytes(const ScanParams& p);
cudaError_t launch_chunked_scan(const ScanParams& p, cudaStream_t s);
// Reads and clears the device error word of the chunked kernels (0 = none).
cudaError_t read_and_clear_device_error(unsigned* code);
// Test hooks of the chunked kernels (gdn_testing.h): wait limit (0 = the
// default) and injected fault, on the current device.
cudaError_t set_test_hooks(unsigned long long wait_ns, int fault);
cudaError_t read_test_hooks(unsigned long long* wait_ns, int* fault);
cudaError_t read_and_clear_qlinear_error(unsigned* code);
// The same for the tcgen05 attention prefill.
cudaError_t read_and_clear_attn_error(unsigned* code);

}  // namespace gdn
