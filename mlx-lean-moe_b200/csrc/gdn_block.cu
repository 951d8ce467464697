// The linear-attention layer's prologue and epilogue around the scan, and
// the forget gate.
//
// Reference (qw/ = src/mlx_lean_moe/model/qwen3_5/):
//   forget_gate           qw/gated_delta.py:14-21
//   _convolve             qw/linear_attention.py:61-79
//   q/k norm, gates       qw/linear_attention.py:104-116
//   _gated_rms_norm       qw/linear_attention.py:22-32, applied at :122-124
//
// Rounding points.  With bfloat16 activations the reference materialises, in
// bfloat16: the conv weight and the conv state cast to the input dtype
// (:69, :72), the conv output, its SiLU (nn.silu is one fused function), the
// rms-normed q/k and their rescaled values (:112-113), beta = sigmoid(b)
// (:116), y cast to z's dtype (:123), the rms-norm output (:28) and the final
// product (:30-32).  The forget gate is computed in float32 (gated_delta.py:18-
// 20) and the scan in float32 (the state is float32).  These kernels compute
// in float32 and round to the activation type at exactly those points (a no-op
// for float32 activations).
#include "gdn_common.cuh"

namespace gdn {
namespace {

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

__global__ void forget_gate_kernel(const void* a, gdn_dtype dt, int64_t a_st, int64_t n, int hv,
                                   const float* A_log, const float* dt_bias, float* g, gdn_gate_kind kind) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= n * hv) return;
  const int64_t t = idx / hv;
  const int h = (int)(idx % hv);
  const int64_t ai = t * a_st + h;
  float av;
  if (dt == GDN_BF16)
    av = __bfloat162float(static_cast<const __nv_bfloat16*>(a)[ai]);
  else if (dt == GDN_F16)
    av = __half2float(static_cast<const __half*>(a)[ai]);
  else
    av = static_cast<const float*>(a)[ai];
  const float lg = -expf(A_log[h]) * softplus_f(av + dt_bias[h]);
  g[idx] = kind == GDN_GATE_LOG ? lg : expf(lg);
}

constexpr int TT = 16;          // tokens per prologue CTA
constexpr int MAXC = 8;         // channels per lane (head width <= 256)
constexpr int MAXK = 8;         // conv kernel width supported

// Sequence containing token t (cu_seqlens sorted, B + 1 entries).
__device__ __forceinline__ int64_t find_seq(const int64_t* cu, int64_t n_tokens, int64_t n_seqs, int64_t t) {
  if (!cu) return t / (n_tokens / n_seqs);
  int64_t lo = 0, hi = n_seqs - 1;
  while (lo < hi) {  // last b with cu[b] <= t, skipping empty sequences
    const int64_t mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

template <typename T, typename TS>
__device__ __forceinline__ float conv_src(const BlockParams& p, int64_t b, int64_t start, int64_t pos, int c) {
  // pos: absolute token index; positions before the sequence start come from
  // that sequence's conv state rows (row K-1 - (start - pos)).
  if (pos >= start) return to_f(static_cast<const T*>(p.mixed)[pos * p.mixed_st + c]);
  if (!p.conv_state_in) return 0.f;
  const int64_t conv_dim = 2LL * p.hk * p.dk + (int64_t)p.hv * p.dv;
  const int64_t row = p.kernel - 1 - (start - pos);
  const float x = to_f(static_cast<const TS*>(p.conv_state_in)[(b * (p.kernel - 1) + row) * conv_dim + c]);
  return round_to<T>(x);
}

// Grid: x = token tiles of TT, y = groups of 4 conv heads (+1 for the gates).
// A conv head is Dk channels of q or k, or Dv channels of v; one warp each.
template <typename T, typename TS>
__global__ void __launch_bounds__(128) block_prologue_kernel(const BlockParams p) {
  griddep_wait();  // launched as a dependent of the kernel before it
  griddep_launch_dependents();
  const int64_t t0 = blockIdx.x * (int64_t)TT;
  const int n_heads = 2 * p.hk + p.hv;
  const int64_t conv_dim = 2LL * p.hk * p.dk + (int64_t)p.hv * p.dv;
  const int64_t off_b = conv_dim + (int64_t)p.hv * p.dv, off_a = off_b + p.hv;

  if (blockIdx.y == gridDim.y - 1) {  // gates
    for (int idx = threadIdx.x; idx < TT * p.hv; idx += blockDim.x) {
      const int64_t t = t0 + idx / p.hv;
      const int h = idx % p.hv;
      if (t >= p.n_tokens) break;
      const T* row = static_cast<const T*>(p.mixed) + t * p.mixed_st;
      const float av = to_f(row[off_a + h]), bv = to_f(row[off_b + h]);
      p.g_log[t * p.hv + h] = -expf(p.A_log[h]) * softplus_f(av + p.dt_bias[h]);
      p.beta[t * p.hv + h] = round_to<T>(sigmoid_f(bv));
    }
    return;
  }

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ch = blockIdx.y * 4 + warp;
  if (ch >= n_heads) return;
  const bool is_q = ch < p.hk, is_k = !is_q && ch < 2 * p.hk;
  const int width = (is_q || is_k) ? p.dk : p.dv;
  const int64_t c0 = ch < 2 * p.hk ? (int64_t)ch * p.dk : 2LL * p.hk * p.dk + (int64_t)(ch - 2 * p.hk) * p.dv;
  const int K = p.kernel;

  float w[MAXC][MAXK];
#pragma unroll
  for (int m = 0; m < MAXC; ++m) {
    const int d = lane + 32 * m;
#pragma unroll
    for (int j = 0; j < MAXK; ++j)
      w[m][j] = (d < width && j < K) ? round_to<T>(p.conv_w[(c0 + d) * K + j]) : 0.f;
  }

  const int64_t t_end = min(t0 + TT, p.n_tokens);
  int64_t b = find_seq(p.cu_seqlens, p.n_tokens, p.n_seqs, t0);
  int64_t s_start, s_end;
  seq_range(p.cu_seqlens, p.n_tokens, p.n_seqs, b, s_start, s_end);
  for (int64_t t = t0; t < t_end; ++t) {
    while (t >= s_end) {  // next non-empty sequence
      ++b;
      seq_range(p.cu_seqlens, p.n_tokens, p.n_seqs, b, s_start, s_end);
    }
    float x[MAXC];
    float ss = 0.f;
#pragma unroll
    for (int m = 0; m < MAXC; ++m) {
      const int d = lane + 32 * m;
      float acc = 0.f;
      if (d < width) {
#pragma unroll
        for (int j = 0; j < MAXK; ++j)
          if (j < K) acc += w[m][j] * conv_src<T, TS>(p, b, s_start, t - (K - 1) + j, (int)(c0 + d));
      }
      const float conv = round_to<T>(acc);
      x[m] = d < width ? round_to<T>(silu_f(conv)) : 0.f;
      ss += x[m] * x[m];
    }
    if (is_q || is_k) {
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / (float)width + 1e-6f);
      const float scale = is_q ? 1.f / (float)p.dk : rsqrtf((float)p.dk);
      T* dst = static_cast<T*>(is_q ? p.q : p.k) + (t * p.hk + (is_q ? ch : ch - p.hk)) * (int64_t)p.dk;
#pragma unroll
      for (int m = 0; m < MAXC; ++m) {
        const int d = lane + 32 * m;
        if (d < width) dst[d] = from_f<T>(round_to<T>(x[m] * inv) * scale);
      }
    } else {
      T* dst = static_cast<T*>(p.v) + (t * p.hv + (ch - 2 * p.hk)) * (int64_t)p.dv;
#pragma unroll
      for (int m = 0; m < MAXC; ++m) {
        const int d = lane + 32 * m;
        if (d < width) dst[d] = from_f<T>(x[m]);
      }
    }
  }
}

// New conv tail per sequence: the last K-1 rows of [conv_state ; qkv_b]
// (qw/linear_attention.py:75-79), in the state's dtype.  One thread per
// (sequence, channel); rows are written in increasing order, and each read
// index is >= the written one, so the update is safe in place.
template <typename T, typename TS>
__global__ void block_conv_tail_kernel(const BlockParams p) {
  griddep_wait();  // launched as a dependent of the kernel before it
  griddep_launch_dependents();
  const int64_t conv_dim = 2LL * p.hk * p.dk + (int64_t)p.hv * p.dv;
  const int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t b = blockIdx.y;
  if (c >= conv_dim) return;
  int64_t start, end;
  seq_range(p.cu_seqlens, p.n_tokens, p.n_seqs, b, start, end);
  const int64_t len = end - start;
  const int km1 = p.kernel - 1;
  TS* out = static_cast<TS*>(p.conv_state_out) + b * km1 * conv_dim;
  const TS* in = static_cast<const TS*>(p.conv_state_in);
  for (int i = 0; i < km1; ++i) {
    const int64_t pos = len - km1 + i;  // position within [conv_state ; qkv] minus (K-1)
    float x;
    if (pos >= 0)
      x = to_f(static_cast<const T*>(p.mixed)[(start + pos) * p.mixed_st + c]);
    else
      x = in ? round_to<T>(to_f(in[(b * km1 + km1 + pos) * conv_dim + c])) : 0.f;
    out[i * conv_dim + c] = from_f<TS>(x);
  }
}

// out = silu(z) * rms_norm(y -> T, norm_w, eps); one warp per (token, head).
template <typename T>
__global__ void __launch_bounds__(256) block_epilogue_kernel(const BlockParams p) {
  griddep_wait();  // launched as a dependent of the kernel before it
  griddep_launch_dependents();
  const int64_t row = blockIdx.x * 8LL + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= p.n_tokens * p.hv) return;
  const int64_t t = row / p.hv;
  const int h = (int)(row % p.hv);
  const int64_t conv_dim = 2LL * p.hk * p.dk + (int64_t)p.hv * p.dv;
  const T* z = static_cast<const T*>(p.mixed) + t * p.mixed_st + conv_dim + (int64_t)h * p.dv;
  const T* y = static_cast<const T*>(p.y) + row * p.dv;  // already in the activation dtype
  float yb[MAXC];
  float ss = 0.f;
#pragma unroll
  for (int m = 0; m < MAXC; ++m) {
    const int d = lane + 32 * m;
    yb[m] = d < p.dv ? to_f(y[d]) : 0.f;
    ss += yb[m] * yb[m];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)p.dv + p.eps);
  T* out = static_cast<T*>(p.out) + row * p.dv;
#pragma unroll
  for (int m = 0; m < MAXC; ++m) {
    const int d = lane + 32 * m;
    if (d < p.dv) {
      const float normed = round_to<T>(yb[m] * inv * p.norm_w[d]);
      out[d] = from_f<T>(silu_f(to_f(z[d])) * normed);
    }
  }
}


// ---------------------------------------------------------------------------
// Vectorized prologue/epilogue for the common shapes (conv kernel <= 4, head
// dims a power of two in [8, 256]).  Same arithmetic and rounding points as
// the general kernels above.
// ---------------------------------------------------------------------------
constexpr int VT = 64;  // tokens per prologue CTA

template <typename T>
__device__ __forceinline__ void load8(const T* src, float (&x)[8]);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* src, float (&x)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(src);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(w[i] << 16);
    x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* src, float (&x)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(src);
  const float4 b = *reinterpret_cast<const float4*>(src + 4);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

template <typename T>
__device__ __forceinline__ void store8(T* dst, const float (&x)[8]);
template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* dst, const float (&x)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
}
template <>
__device__ __forceinline__ void store8<float>(float* dst, const float (&x)[8]) {
  *reinterpret_cast<float4*>(dst) = make_float4(x[0], x[1], x[2], x[3]);
  *reinterpret_cast<float4*>(dst + 4) = make_float4(x[4], x[5], x[6], x[7]);
}

// A raw 8-channel row as loaded from global memory (16 bytes of bf16 or 32
// bytes of float), converted to floats later.
template <typename T>
struct Raw8;
template <>
struct Raw8<__nv_bfloat16> {
  uint4 u;
  __device__ __forceinline__ void load(const __nv_bfloat16* src) { u = __ldg(reinterpret_cast<const uint4*>(src)); }
  __device__ __forceinline__ void to_float(float (&x)[8]) const {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __uint_as_float(w[i] << 16);
      x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
};
template <>
struct Raw8<float> {
  float4 a, b;
  __device__ __forceinline__ void load(const float* src) {
    a = __ldg(reinterpret_cast<const float4*>(src));
    b = __ldg(reinterpret_cast<const float4*>(src) + 1);
  }
  __device__ __forceinline__ void to_float(float (&x)[8]) const {
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  }
};

// One row (8 channels starting at c) of the conv input at absolute position
// pos for sequence b starting at `start`: the projection row, or the
// sequence's conv state for positions before its start.
template <typename T, typename TS>
__device__ __forceinline__ void conv_row(const BlockParams& p, int64_t conv_dim, int64_t b, int64_t start,
                                         int64_t pos, int c, float (&x)[8]) {
  if (pos >= start) {
    load8<T>(static_cast<const T*>(p.mixed) + pos * p.mixed_st + c, x);
    return;
  }
  if (!p.conv_state_in) {
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = 0.f;
    return;
  }
  const int64_t row = p.kernel - 1 - (start - pos);
  const TS* src = static_cast<const TS*>(p.conv_state_in) + (b * (p.kernel - 1) + row) * conv_dim + c;
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = round_to<T>(to_f(src[i]));
}

// Grid: x = token tiles of VT, y = channel blocks of 2048 (+1 for the gates).
// Thread: 8 consecutive channels; a warp covers 256 channels, so a q/k head
// of Dk channels is Dk/8 consecutive lanes (Dk a power of two <= 256).
template <typename T, typename TS, int K>
__global__ void __launch_bounds__(256) block_prologue_fast_kernel(const BlockParams p) {
  griddep_wait();  // launched as a dependent of the kernel before it
  griddep_launch_dependents();
  const int64_t t0 = blockIdx.x * (int64_t)VT;
  const int64_t t_end = min(t0 + VT, p.n_tokens);
  const int64_t conv_dim = 2LL * p.hk * p.dk + (int64_t)p.hv * p.dv;
  if (blockIdx.y == gridDim.y - 1) {  // gates
    const int64_t off_b = conv_dim + (int64_t)p.hv * p.dv, off_a = off_b + p.hv;
    for (int idx = threadIdx.x; idx < VT * p.hv; idx += blockDim.x) {
      const int64_t t = t0 + idx / p.hv;
      const int h = idx % p.hv;
      if (t >= p.n_tokens) break;
      const T* row = static_cast<const T*>(p.mixed) + t * p.mixed_st;
      const float av = to_f(row[off_a + h]), bv = to_f(row[off_b + h]);
      p.g_log[t * p.hv + h] = -expf(p.A_log[h]) * softplus_f(av + p.dt_bias[h]);
      p.beta[t * p.hv + h] = round_to<T>(sigmoid_f(bv));
    }
    return;
  }
  // Lanes past the last channel stay in the loop (without loads or stores)
  // so that every shuffle below has its full warp.
  const int c_raw = (int)(blockIdx.y * 2048 + threadIdx.x * 8);
  const bool active = c_raw < conv_dim;  // whole 8-groups only (conv_dim % 8 == 0)
  const int c = active ? c_raw : 0;
  const int64_t key_dim = (int64_t)p.hk * p.dk;
  const bool is_q = c < key_dim, is_k = !is_q && c < 2 * key_dim;
  const int group = (is_q || is_k) ? p.dk / 8 : 32;  // lanes sharing one q/k head
  const bool qk_warp = __any_sync(0xffffffffu, is_q || is_k);

  float w[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) w[i][j] = j < K ? round_to<T>(p.conv_w[(int64_t)(c + i) * K + j]) : 0.f;

  int64_t b = find_seq(p.cu_seqlens, p.n_tokens, p.n_seqs, t0);
  int64_t s_start, s_end;
  seq_range(p.cu_seqlens, p.n_tokens, p.n_seqs, b, s_start, s_end);
  // win[j] = conv input at position t - (K-1) + j, j < K-1 (the history)
  float win[K > 1 ? K - 1 : 1][8];
  auto reset = [&](int64_t t) {
#pragma unroll
    for (int j = 0; j < K - 1; ++j) conv_row<T, TS>(p, conv_dim, b, s_start, t - (K - 1) + j, c, win[j]);
  };
  reset(t0);
  const float qscale = 1.f / (float)p.dk, kscale = rsqrtf((float)p.dk);
  const T* src = static_cast<const T*>(p.mixed) + c;
  // Rows t .. t+PF-1 are loaded before row t is used, so the loads run ahead
  // of the arithmetic and the stores.
  constexpr int PF = 4;
  Raw8<T> ring[PF];
#pragma unroll
  for (int u = 0; u < PF; ++u)
    if (active && t0 + u < t_end) ring[u].load(src + (t0 + u) * p.mixed_st);
  for (int64_t tb = t0; tb < t_end; tb += PF) {
#pragma unroll
    for (int u = 0; u < PF; ++u) {
      const int64_t t = tb + u;
      if (t >= t_end) break;
      if (t >= s_end) {  // next (non-empty) sequence: fresh history from its conv state
        do {
          ++b;
          seq_range(p.cu_seqlens, p.n_tokens, p.n_seqs, b, s_start, s_end);
        } while (t >= s_end);
        reset(t);
      }
      float cur[8];
      ring[u].to_float(cur);
      if (active && t + PF < t_end) ring[u].load(src + (t + PF) * p.mixed_st);
      float x[8];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {  // channel pairs: packed FMAs, the scalar order per channel
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < K - 1; ++j)
          acc = ffma2(make_float2(w[i][j], w[i + 1][j]), make_float2(win[j][i], win[j][i + 1]), acc);
        acc = ffma2(make_float2(w[i][K - 1], w[i + 1][K - 1]), make_float2(cur[i], cur[i + 1]), acc);
        x[i] = acc.x;
        x[i + 1] = acc.y;
      }
      round8<T>(x);  // the conv output, then SiLU of it, in the activation dtype
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = silu_fast(x[i]);
      round8<T>(x);
      // q/k rms-norm: reduce over the lanes of this head (all lanes of a
      // warp holding any q/k channel shuffle; v-only warps skip it).
      float ss = 0.f;
      if (qk_warp) {
#pragma unroll
        for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
          const float o = __shfl_xor_sync(0xffffffffu, ss, off);
          if (off < group) ss += o;
        }
      }
      if (is_q || is_k) {
        const float inv = rsqrtf(ss / (float)p.dk + 1e-6f);
        const float scale = is_q ? qscale : kscale;
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const float2 r = fmul2(make_float2(x[i], x[i + 1]), make_float2(inv, inv));
          x[i] = r.x;
          x[i + 1] = r.y;
        }
        round8<T>(x);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const float2 r = fmul2(make_float2(x[i], x[i + 1]), make_float2(scale, scale));
          x[i] = r.x;
          x[i + 1] = r.y;
        }
        round8<T>(x);
        T* dst = static_cast<T*>(is_q ? p.q : p.k) + t * key_dim + (is_q ? c : c - key_dim);
        if (active) store8<T>(dst, x);
      } else {
        T* dst = static_cast<T*>(p.v) + t * (int64_t)p.hv * p.dv + (c - 2 * key_dim);
        if (active) store8<T>(dst, x);
      }
      // slide the history window
#pragma unroll
      for (int j = 0; j + 1 < K - 1; ++j)
#pragma unroll
        for (int i = 0; i < 8; ++i) win[j][i] = win[j + 1][i];
      if constexpr (K > 1) {
#pragma unroll
        for (int i = 0; i < 8; ++i) win[K - 2][i] = cur[i];
      }
    }
  }
}

// out = silu(z) * rms_norm(y -> T, norm_w, eps); Dv/8 lanes per (token, head)
// row, 8 values per lane.
template <typename T>
__global__ void __launch_bounds__(256) block_epilogue_fast_kernel(const BlockParams p) {
  griddep_wait();  // launched as a dependent of the kernel before it
  griddep_launch_dependents();
  const int lanes = p.dv / 8;
  const int64_t gtid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t row = gtid / lanes;
  const int d0 = (int)(gtid % lanes) * 8;
  const bool valid = row < p.n_tokens * p.hv;
  const int64_t rr = valid ? row : 0;
  const int64_t t = rr / p.hv;
  const int h = (int)(rr % p.hv);
  const int64_t conv_dim = 2LL * p.hk * p.dk + (int64_t)p.hv * p.dv;
  float y[8], z[8], w[8];
  load8<T>(static_cast<const T*>(p.y) + rr * p.dv + d0, y);  // already in the activation dtype
  load8<T>(static_cast<const T*>(p.mixed) + t * p.mixed_st + conv_dim + (int64_t)h * p.dv + d0, z);
  load8<float>(p.norm_w + d0, w);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += y[i] * y[i];
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, ss, off);
    if (off < lanes) ss += o;
  }
  const float inv = rsqrtf(ss / (float)p.dv + p.eps);
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = y[i] * inv * w[i];
  round8<T>(o);
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] *= silu_fast(z[i]);
  if (valid) store8<T>(static_cast<T*>(p.out) + rr * p.dv + d0, o);
}

// ------------------------------------------------------------------ decode
// Every sequence one token (decode through the layer): the whole block for
// one (sequence, value head) in one CTA of 384 threads, used when the new
// conv tail goes to a buffer of its own.
//  phase 1, a thread per channel of the head (warps 0-3 q, 4-7 k, 8-11 v):
//    the causal conv over the conv state and the token, SiLU, the q/k RMS
//    norms and scales, rounded where block_prologue_fast_kernel rounds; the
//    new conv tail of those channels (q/k channels by the first value head of
//    their group only); the gates (thread 0).
//  phase 2, warps 0-7: the state update of decode_kernel, a state row over 8
//    lanes, the state loads issued before phase 1.
//  phase 3, warps 0-3: the gated RMS norm of block_epilogue_fast_kernel.
constexpr int kDecDim = 128;  // Dk = Dv

template <typename T, typename TS, int K>
__global__ void __launch_bounds__(384) block_decode_kernel(const BlockParams p, const float* state_in,
                                                           float* state_out) {
  griddep_wait();  // launched as a dependent of the kernel before it
  griddep_launch_dependents();
  constexpr int LPR = 8, VEC = 4, RPG = 4, ITER = 4;  // 8 warps x 4 rows x 4 passes = 128 rows
  __shared__ __align__(16) float qs[kDecDim];
  __shared__ __align__(16) float ks[kDecDim];
  __shared__ float vs[kDecDim], ys[kDecDim];
  __shared__ float red[8];
  __shared__ float gate[2];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x;
  const int64_t b = blockIdx.y;  // sequence b is token b
  const int group = p.hv / p.hk, kh = h / group;
  const int64_t key_dim = (int64_t)p.hk * kDecDim;
  const int64_t conv_dim = 2 * key_dim + (int64_t)p.hv * kDecDim;
  const T* mrow = static_cast<const T*>(p.mixed) + b * p.mixed_st;
  const int64_t head_off = (b * p.hv + h) * (int64_t)kDecDim * kDecDim;
  const int grp = lane / LPR, l = lane % LPR;
  const int row0 = warp * (RPG * ITER) + grp;

  float4 s[ITER][VEC];
  if (warp < 8) {
#pragma unroll
    for (int i = 0; i < ITER; ++i)
#pragma unroll
      for (int j = 0; j < VEC; ++j)
        s[i][j] = state_in ? *reinterpret_cast<const float4*>(state_in + head_off +
                                                               (int64_t)(row0 + i * RPG) * kDecDim + (j * LPR + l) * 4)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
  }

  // phase 1
  const int part = tid >> 7, i = tid & 127;  // 0: q, 1: k, 2: v
  const int64_t c = part == 0 ? kh * kDecDim + i : part == 1 ? key_dim + kh * kDecDim + i
                                                             : 2 * key_dim + (int64_t)h * kDecDim + i;
  float win[K > 1 ? K - 1 : 1];
#pragma unroll
  for (int j = 0; j < K - 1; ++j)
    win[j] = p.conv_state_in
                 ? round_to<T>(to_f(static_cast<const TS*>(p.conv_state_in)[(b * (K - 1) + j) * conv_dim + c]))
                 : 0.f;
  const float cur = to_f(mrow[c]);
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < K - 1; ++j) acc += round_to<T>(p.conv_w[c * K + j]) * win[j];
  acc += round_to<T>(p.conv_w[c * K + K - 1]) * cur;
  float x = round_to<T>(silu_fast(round_to<T>(acc)));
  if constexpr (K > 1) {
    if (part == 2 || h % group == 0) {
      TS* tail = static_cast<TS*>(p.conv_state_out) + b * (K - 1) * conv_dim + c;
#pragma unroll
      for (int r = 0; r < K - 1; ++r) tail[r * conv_dim] = from_f<TS>(r < K - 2 ? win[r + 1] : cur);
    }
  }
  if (tid == 0) {
    const int64_t off_b = conv_dim + (int64_t)p.hv * kDecDim, off_a = off_b + p.hv;
    const float av = to_f(mrow[off_a + h]), bv = to_f(mrow[off_b + h]);
    gate[0] = expf(-expf(p.A_log[h]) * softplus_f(av + p.dt_bias[h]));
    gate[1] = round_to<T>(sigmoid_f(bv));
  }
  float ss = part < 2 ? x * x : 0.f;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0 && warp < 8) red[warp] = ss;
  __syncthreads();
  if (part < 2) {
    const float tot = red[part * 4] + red[part * 4 + 1] + red[part * 4 + 2] + red[part * 4 + 3];
    const float inv = rsqrtf(tot / (float)kDecDim + 1e-6f);
    x = round_to<T>(round_to<T>(x * inv) * (part == 0 ? 1.f / (float)kDecDim : rsqrtf((float)kDecDim)));
    (part == 0 ? qs : ks)[i] = x;
  } else {
    vs[i] = x;
  }
  __syncthreads();

  // phase 2
  if (warp < 8) {
    const float gv = gate[0], bv = gate[1];
    float4 kq[VEC], qq[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      kq[j] = *reinterpret_cast<const float4*>(ks + (j * LPR + l) * 4);
      qq[j] = *reinterpret_cast<const float4*>(qs + (j * LPR + l) * 4);
    }
    float* sout = state_out + head_off;
#pragma unroll
    for (int it = 0; it < ITER; ++it) {
      const int row = row0 + it * RPG;
      float r = 0.f;
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        s[it][j] = s[it][j] * gv;
        r += dot4(s[it][j], kq[j]);
      }
#pragma unroll
      for (int off = LPR / 2; off >= 1; off >>= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
      const float d = (vs[row] - r) * bv;
      float y = 0.f;
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        s[it][j].x += kq[j].x * d;
        s[it][j].y += kq[j].y * d;
        s[it][j].z += kq[j].z * d;
        s[it][j].w += kq[j].w * d;
        y += dot4(s[it][j], qq[j]);
        *reinterpret_cast<float4*>(sout + (int64_t)row * kDecDim + (j * LPR + l) * 4) = s[it][j];
      }
#pragma unroll
      for (int off = LPR / 2; off >= 1; off >>= 1) y += __shfl_xor_sync(0xffffffffu, y, off);
      if (l == 0) ys[row] = round_to<T>(y);
    }
  }
  __syncthreads();

  // phase 3
  float y = 0.f;
  if (warp < 4) {
    y = ys[tid];
    float sq = y * y;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
    if (lane == 0) red[warp] = sq;
  }
  __syncthreads();
  if (warp < 4) {
    const float inv = rsqrtf((red[0] + red[1] + red[2] + red[3]) / (float)kDecDim + p.eps);
    const float o = round_to<T>(y * inv * p.norm_w[tid]);
    const float z = to_f(mrow[conv_dim + (int64_t)h * kDecDim + tid]);
    static_cast<T*>(p.out)[(b * p.hv + h) * (int64_t)kDecDim + tid] = from_f<T>(o * silu_fast(z));
  }
}

template <typename T, typename TS>
cudaError_t decode_t(const BlockParams& p, const float* state_in, float* state_out, cudaStream_t s) {
  const dim3 grid((unsigned)p.hv, (unsigned)p.n_seqs);
  switch (p.kernel) {
    case 1: return launch_dependent(block_decode_kernel<T, TS, 1>, grid, dim3(384), 0, s, p, state_in, state_out);
    case 2: return launch_dependent(block_decode_kernel<T, TS, 2>, grid, dim3(384), 0, s, p, state_in, state_out);
    case 3: return launch_dependent(block_decode_kernel<T, TS, 3>, grid, dim3(384), 0, s, p, state_in, state_out);
    default: return launch_dependent(block_decode_kernel<T, TS, 4>, grid, dim3(384), 0, s, p, state_in, state_out);
  }
}

bool pow2_in(int x, int lo, int hi) { return x >= lo && x <= hi && (x & (x - 1)) == 0; }

bool fast_shapes(const BlockParams& p) {
  return p.kernel >= 1 && p.kernel <= 4 && pow2_in(p.dk, 8, 256) && pow2_in(p.dv, 8, 256) && p.mixed_st % 8 == 0 &&
         (reinterpret_cast<uintptr_t>(p.mixed) & 15u) == 0 && (reinterpret_cast<uintptr_t>(p.norm_w) & 15u) == 0;
}

template <typename T, typename TS, int K>
cudaError_t launch_prologue_fast(dim3 grid, const BlockParams& p, cudaStream_t s) {
  return launch_dependent(block_prologue_fast_kernel<T, TS, K>, grid, dim3(256), 0, s, p);
}

template <typename T, typename TS>
cudaError_t prologue_t(const BlockParams& p, cudaStream_t s) {
  if (fast_shapes(p)) {
    const int64_t conv_dim = 2LL * p.hk * p.dk + (int64_t)p.hv * p.dv;
    const int64_t gx = (p.n_tokens + VT - 1) / VT;
    if (gx == 0) return cudaSuccess;
    dim3 grid((unsigned)gx, (unsigned)((conv_dim + 2047) / 2048 + 1));
    switch (p.kernel) {
      case 1: return launch_prologue_fast<T, TS, 1>(grid, p, s);
      case 2: return launch_prologue_fast<T, TS, 2>(grid, p, s);
      case 3: return launch_prologue_fast<T, TS, 3>(grid, p, s);
      default: return launch_prologue_fast<T, TS, 4>(grid, p, s);
    }
  }
  const int n_heads = 2 * p.hk + p.hv;
  const int64_t gx = (p.n_tokens + TT - 1) / TT;
  if (gx == 0) return cudaSuccess;
  dim3 grid((unsigned)gx, (unsigned)((n_heads + 3) / 4 + 1));
  return launch_dependent(block_prologue_kernel<T, TS>, grid, dim3(128), 0, s, p);
}

template <typename T, typename TS>
cudaError_t tail_t(const BlockParams& p, cudaStream_t s) {
  const int64_t conv_dim = 2LL * p.hk * p.dk + (int64_t)p.hv * p.dv;
  if (p.kernel <= 1 || p.n_seqs == 0) return cudaSuccess;
  dim3 grid((unsigned)((conv_dim + 255) / 256), (unsigned)p.n_seqs);
  return launch_dependent(block_conv_tail_kernel<T, TS>, grid, dim3(256), 0, s, p);
}

}  // namespace

cudaError_t launch_forget_gate(const void* a, gdn_dtype dt, int64_t a_st, int64_t n, int hv, const float* A_log,
                               const float* dt_bias, float* g, gdn_gate_kind kind, cudaStream_t s) {
  const int64_t total = n * hv;
  if (total == 0) return cudaSuccess;
  forget_gate_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(a, dt, a_st, n, hv, A_log, dt_bias, g, kind);
  return cudaGetLastError();
}

cudaError_t launch_block_prologue(const BlockParams& p, cudaStream_t s) {
  const bool st_bf = p.conv_state_dtype == GDN_BF16;
  if (p.act_dtype == GDN_BF16)
    return st_bf ? prologue_t<__nv_bfloat16, __nv_bfloat16>(p, s) : prologue_t<__nv_bfloat16, float>(p, s);
  return st_bf ? prologue_t<float, __nv_bfloat16>(p, s) : prologue_t<float, float>(p, s);
}

cudaError_t launch_block_conv_tail(const BlockParams& p, cudaStream_t s) {
  const bool st_bf = p.conv_state_dtype == GDN_BF16;
  if (p.act_dtype == GDN_BF16)
    return st_bf ? tail_t<__nv_bfloat16, __nv_bfloat16>(p, s) : tail_t<__nv_bfloat16, float>(p, s);
  return st_bf ? tail_t<float, __nv_bfloat16>(p, s) : tail_t<float, float>(p, s);
}

cudaError_t launch_block_epilogue(const BlockParams& p, cudaStream_t s) {
  const int64_t rows = p.n_tokens * p.hv;
  if (rows == 0) return cudaSuccess;
  if (fast_shapes(p)) {
    const int64_t threads = rows * (p.dv / 8);
    const unsigned grid = (unsigned)((threads + 255) / 256);
    if (p.act_dtype == GDN_BF16)
      return launch_dependent(block_epilogue_fast_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, s, p);
    return launch_dependent(block_epilogue_fast_kernel<float>, dim3(grid), dim3(256), 0, s, p);
  }
  const unsigned grid = (unsigned)((rows + 7) / 8);
  if (p.act_dtype == GDN_BF16)
    return launch_dependent(block_epilogue_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, s, p);
  return launch_dependent(block_epilogue_kernel<float>, dim3(grid), dim3(256), 0, s, p);
}

bool block_decode_supported(const BlockParams& p, const float* state_in, const float* state_out) {
  if (p.n_tokens != p.n_seqs || p.n_seqs < 1 || p.cu_seqlens || p.dk != kDecDim || p.dv != kDecDim) return false;
  if (p.kernel < 1 || p.kernel > 4 || p.hv % p.hk || p.n_seqs > 65535) return false;
  if ((reinterpret_cast<uintptr_t>(state_in) | reinterpret_cast<uintptr_t>(state_out)) & 15u) return false;
  if (p.kernel > 1 && p.conv_state_in) {  // the conv tail must not overwrite state that other CTAs still read
    const size_t bytes = (size_t)p.n_seqs * (p.kernel - 1) * (2 * (size_t)p.hk * p.dk + (size_t)p.hv * p.dv) *
                         (p.conv_state_dtype == GDN_BF16 ? 2 : 4);
    const uintptr_t in = reinterpret_cast<uintptr_t>(p.conv_state_in), out = reinterpret_cast<uintptr_t>(p.conv_state_out);
    if (in < out + bytes && out < in + bytes) return false;
  }
  return true;
}

cudaError_t launch_block_decode(const BlockParams& p, const float* state_in, float* state_out, cudaStream_t s) {
  const bool st_bf = p.conv_state_dtype == GDN_BF16;
  if (p.act_dtype == GDN_BF16)
    return st_bf ? decode_t<__nv_bfloat16, __nv_bfloat16>(p, state_in, state_out, s)
                 : decode_t<__nv_bfloat16, float>(p, state_in, state_out, s);
  return st_bf ? decode_t<float, __nv_bfloat16>(p, state_in, state_out, s) : decode_t<float, float>(p, state_in, state_out, s);
}

}  // namespace gdn
