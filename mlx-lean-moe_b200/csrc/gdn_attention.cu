// The softmax-attention layer's core (the reference's Qwen3_5Attention
// between its projections, qw/attention.py:56-96, with the GrowingKVCache of
// cache/kv_cache.py): q/k RMS norms with weights, rotary embedding of the
// leading rotary_dim features (model/rope.py: feature i pairs with
// i + rotary_dim / 2, angle = position * base^(-2i / rotary_dim)), the append
// of this call's keys and values to a head-major cache, grouped-query
// attention with the causal mask aligned to the newest query, and the
// output gate sigmoid(gate) carried in q_proj's second half.
//
// attn_prep_kernel     one CTA per token, a warp per row of q / k / v heads
//                      (four rows per warp for prefill): the
//                      norms and the rotation in float32, rounded to the
//                      activation dtype where the reference materializes
//                      arrays; q to the workspace, k and v into the cache.
//                      Rotation angles are reduced modulo 2 pi in double
//                      precision before sincosf, so long positions keep
//                      their accuracy.
// attn_fwd_kernel      flash-style attention on the CUDA cores in float32:
//                      one CTA per (kRows query rows of one key/value head,
//                      key split); its eight warps share each 32-key K/V tile
//                      (cp.async, double-buffered) and own one row each, with
//                      their own running max and sum (lane = key for the
//                      scores, lane = features for the output).  One split finishes the
//                      rows (normalization, gate, output); several write
//                      partial (max, sum, output) rows that
// attn_combine_kernel  adds up, then gates and writes.
// attn_tc_kernel       bf16 prefill (calls with enough rows for one key
//                      split), head_dim 128 or 256: tcgen05 MMAs into TMEM,
//                      Q, K and V by TMA; see its comment below.
// attn_mma_kernel      the same for head_dim 64, or when the tensor maps
//                      cannot be made: mma.sync on the tensor cores.
// attn_dec_mma_kernel  bf16 decode (one token, a key/value head's query
//                      heads within 16 rows) on the tensor cores, one warp
//                      per key split, into the combine.
//
// The attention and combine kernels are launched as programmatic dependents
// of the kernel before them: they start while it finishes, and the
// attention kernel fetches keys cached by earlier calls before it waits for
// the prep kernel's output.
#include <cuda_bf16.h>

#include <cmath>
#include <cstring>
#include <type_traits>

#include <cudaTypedefs.h>

#include "gdn_api.h"
#include "gdn_common.cuh"
#include "gdn_sm100.cuh"

namespace gdn {
namespace {

constexpr int kRows = 8;        // query rows (token x head) per CTA
constexpr int kWarps = 8;      // one query row each
constexpr int kKeyTile = 32;    // keys per warp step
constexpr int kMaxHeadDim = 256;

struct AttnParams {
  int64_t n_tokens, cache_len, offset;  // offset = cache_len - n_tokens: position of the first new token
  int heads, kv_heads, head_dim, rotary_dim, group;  // group = heads / kv_heads
  float eps, scale;
  double inv_freq[kMaxHeadDim / 2];     // rope_base^(-2i / rotary_dim), from the host in double
  const void* qg;
  int64_t qg_st;
  const void* k_new;
  int64_t k_st;
  const void* v_new;
  int64_t v_st;
  const float* q_norm;
  const float* k_norm;
  void* k_cache;
  void* v_cache;
  int64_t cache_sh;                     // elements between heads of the caches (capacity * head_dim)
  void* q_ws;                           // [n_tokens, heads, head_dim] in the activation dtype
  float* part;                          // [splits, n_tokens * heads, head_dim + 4]: output, max, sum, pad
  int splits;
  void* out;
  int64_t out_st;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ------------------------------------------------------------------ prep
// One CTA per token.  Its threads first compute the token's (cos, sin) per
// rotary frequency into shared memory (once for all of its heads); then each
// warp takes head rows of the token: rows [0, heads) are queries, then the
// kv_heads keys, then the kv_heads values, each lane holding head_dim / 32
// consecutive features.  The norm reduces by shuffles; the rotation reads its
// partner features from the warp's row in shared memory.  A warp takes RPW
// rows (rows warp, warp + nwarps, ...), all loaded before the angles are
// computed: RPW = 1 (a warp per row) for calls with few tokens, where the
// latency of one CTA matters; RPW = 4 for prefill, where CTAs of fewer warps
// fit more per SM and keep more loads in flight.  Further rows, if any, go
// one at a time.  VEC: every row start is aligned to its lane's run of
// features (up to 16 bytes), so each lane moves its run in vector accesses.
constexpr int kPrepMaxWarps = 32;

template <int B>
struct VecOf;
template <>
struct VecOf<16> { using type = uint4; };
template <>
struct VecOf<8> { using type = uint2; };
template <>
struct VecOf<4> { using type = uint32_t; };
template <>
struct VecOf<2> { using type = uint16_t; };

// N consecutive elements of T (vector accesses of up to 16 bytes when VEC).
template <typename T, int N, bool VEC>
__device__ __forceinline__ void ld_run(const T* src, float (&x)[N]) {
  alignas(16) T v[N];
  if constexpr (VEC) {
    constexpr int B = N * (int)sizeof(T), W = B >= 16 ? 16 : B;
    using V = typename VecOf<W>::type;
#pragma unroll
    for (int i = 0; i < B / W; ++i) reinterpret_cast<V*>(v)[i] = reinterpret_cast<const V*>(src)[i];
  } else {
#pragma unroll
    for (int e = 0; e < N; ++e) v[e] = src[e];
  }
#pragma unroll
  for (int e = 0; e < N; ++e) x[e] = to_f(v[e]);
}

template <typename T, int N, bool VEC>
__device__ __forceinline__ void st_run(T* dst, const float (&x)[N]) {
  alignas(16) T v[N];
  if constexpr (std::is_same<T, __nv_bfloat16>::value && N % 2 == 0) {
#pragma unroll
    for (int e = 0; e < N; e += 2) *reinterpret_cast<uint32_t*>(&v[e]) = cvt_bf16x2(x[e], x[e + 1]);
  } else {
#pragma unroll
    for (int e = 0; e < N; ++e) v[e] = from_f<T>(x[e]);
  }
  if constexpr (VEC) {
    constexpr int B = N * (int)sizeof(T), W = B >= 16 ? 16 : B;
    using V = typename VecOf<W>::type;
#pragma unroll
    for (int i = 0; i < B / W; ++i) reinterpret_cast<V*>(dst)[i] = reinterpret_cast<const V*>(v)[i];
  } else {
#pragma unroll
    for (int e = 0; e < N; ++e) dst[e] = v[e];
  }
}

// Rounds N floats to the precision of T (in pairs for bf16).
template <typename T, int N>
__device__ __forceinline__ void round_run(float (&x)[N]) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value && N % 2 == 0) {
#pragma unroll
    for (int e = 0; e < N; e += 2) round2_bf16(x[e], x[e + 1]);
  } else {
#pragma unroll
    for (int e = 0; e < N; ++e) x[e] = round_to<T>(x[e]);
  }
}

// The rotation angle pos * f reduced to about [-pi, pi] in double: k = the
// integer nearest ang / (2 pi), then ang - k * 2 pi with 2 pi split in two
// doubles (C1 = 2 pi rounded to double, C2 = 2 pi - C1), each product taken
// inside one fused multiply-add (Cody and Waite's additive range reduction).
__device__ __forceinline__ float rope_angle(int64_t pos, double f) {
  const double ang = (double)pos * f;
  const double k = rint(ang * 0.15915494309189535);
  double r = fma(-k, 6.283185307179586, ang);
  r = fma(-k, 2.4492935982947064e-16, r);
  return (float)r;
}

template <typename T, int HD, bool VEC, int RPW>
__global__ void __launch_bounds__(RPW == 1 ? kPrepMaxWarps * 32 : 256) attn_prep_kernel(const AttnParams p) {
  constexpr int DPL = HD / 32;
  __shared__ float xs[RPW == 1 ? kPrepMaxWarps : 8][HD];
  __shared__ float2 rot[HD / 2];  // (cos, sin) of this token's angle per frequency
  griddep_launch_dependents();    // the attention kernel waits for this grid before it reads q or the new keys
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int64_t t = blockIdx.x;
  const int64_t pos = p.offset + t;
  const int rows = p.heads + 2 * p.kv_heads, half = p.rotary_dim / 2, d0 = lane * DPL;
  // row r of this token
  auto load = [&](int r, float (&x)[DPL]) {
    if (r < p.heads)
      ld_run<T, DPL, VEC>(static_cast<const T*>(p.qg) + t * p.qg_st + (int64_t)r * 2 * HD + d0, x);
    else if (r < p.heads + p.kv_heads)
      ld_run<T, DPL, VEC>(static_cast<const T*>(p.k_new) + t * p.k_st + (int64_t)(r - p.heads) * HD + d0, x);
    else
      ld_run<T, DPL, VEC>(
          static_cast<const T*>(p.v_new) + t * p.v_st + (int64_t)(r - p.heads - p.kv_heads) * HD + d0, x);
  };
  float* xr = xs[warp];
  // row r: RMS norm with its weights and rotation (queries, keys) or a copy into the cache (values)
  auto process = [&](int row, float (&x)[DPL]) {
    if (row >= p.heads + p.kv_heads) {
      st_run<T, DPL, VEC>(static_cast<T*>(p.v_cache) + (row - p.heads - p.kv_heads) * p.cache_sh + pos * HD + d0,
                          x);
      return;
    }
    const bool is_q = row < p.heads;
    float w[DPL];
    ld_run<float, DPL, VEC>((is_q ? p.q_norm : p.k_norm) + d0, w);
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) ss += x[e] * x[e];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.f / sqrtf(ss / (float)HD + p.eps);
#pragma unroll
    for (int e = 0; e < DPL; ++e) x[e] = x[e] * inv * w[e];
    round_run<T, DPL>(x);
    __syncwarp();  // the previous row's partner reads are done
#pragma unroll
    for (int e = 0; e < DPL; ++e) xr[d0 + e] = x[e];
    __syncwarp();
    float y[DPL];
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
      const int d = d0 + e;
      y[e] = x[e];
      if (d < p.rotary_dim) {
        const float2 cs = rot[d < half ? d : d - half];
        y[e] = d < half ? x[e] * cs.x - xr[d + half] * cs.y : x[e] * cs.x + xr[d - half] * cs.y;
      }
    }
    T* dst = is_q ? static_cast<T*>(p.q_ws) + (t * p.heads + row) * HD + d0
                  : static_cast<T*>(p.k_cache) + (row - p.heads) * p.cache_sh + pos * HD + d0;
    st_run<T, DPL, VEC>(dst, y);
  };
  float x[RPW][DPL];
#pragma unroll
  for (int i = 0; i < RPW; ++i)  // in flight while the angles are computed
    if (warp + i * nwarps < rows) load(warp + i * nwarps, x[i]);
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float sn, cs;
    sincosf(rope_angle(pos, p.inv_freq[i]), &sn, &cs);
    rot[i] = make_float2(cs, sn);
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < RPW; ++i)
    if (warp + i * nwarps < rows) process(warp + i * nwarps, x[i]);
  for (int row = warp + RPW * nwarps; row < rows; row += nwarps) {
    float x1[DPL];
    load(row, x1);
    process(row, x1);
  }
}

// ------------------------------------------------------------ attention
// Shared memory: the CTA's q rows (float32), then two buffers of a 32-key K
// tile (activation dtype, each row padded by 16 bytes: an odd 16-byte stride
// keeps the lanes' reads of their own key rows free of bank conflicts) and
// of the V tile, then each warp's probabilities.
template <typename T, int HD>
struct AttnSmem {
  static constexpr int kVec = 16 / (int)sizeof(T);                 // elements per 16-byte vector
  static constexpr int kKRow = HD + kVec;                          // padded K row (elements)
  static constexpr size_t kQ = (size_t)kRows * HD * 4;
  static constexpr size_t kKT = (size_t)kKeyTile * kKRow * sizeof(T);  // one K tile
  static constexpr size_t kVT = (size_t)kKeyTile * HD * sizeof(T);     // one V tile
  static constexpr size_t kP = (size_t)kRows * kKeyTile * 4;
  static constexpr size_t kBytes = kQ + 2 * (kKT + kVT) + kP;
};

template <typename T>
__device__ __forceinline__ void load_vec(const T* src, float* dst, int n) {
  // n consecutive elements (n * sizeof(T) a multiple of 16, src 16-byte aligned)
  for (int i = 0; i < n; i += 16 / (int)sizeof(T)) {
    const uint4 u = *reinterpret_cast<const uint4*>(src + i);
    if constexpr (sizeof(T) == 4) {
      dst[i] = __uint_as_float(u.x);
      dst[i + 1] = __uint_as_float(u.y);
      dst[i + 2] = __uint_as_float(u.z);
      dst[i + 3] = __uint_as_float(u.w);
    } else {
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        dst[i + 2 * j] = __uint_as_float(w[j] << 16);
        dst[i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
      }
    }
  }
}

// One CTA: kRows query rows of one key/value head and one key split; the
// eight warps share each K/V tile (cp.async, double-buffered, rows past the
// split's end zero-filled) and each owns kRows / kWarps rows with its own
// running max and sum.  Launched as a programmatic dependent of the prep
// kernel: the first tile, when it holds only keys cached by earlier calls, is
// requested before the wait for the prep kernel's q rows and new keys.
template <typename T, int HD>
__global__ void __launch_bounds__(kWarps * 32) attn_fwd_kernel(const AttnParams p) {
  using SM = AttnSmem<T, HD>;
  constexpr int DPL = HD / 32;            // output features per lane (consecutive)
  constexpr int RPW = kRows / kWarps;     // query rows per warp
  constexpr int VPR = HD / SM::kVec;      // 16-byte vectors per row
  extern __shared__ __align__(16) unsigned char smem[];
  float* qs = reinterpret_cast<float*>(smem);
  unsigned char* tiles = smem + SM::kQ;  // K[0], V[0], K[1], V[1]
  float* ps_all = reinterpret_cast<float*>(smem + SM::kQ + 2 * (SM::kKT + SM::kVT));
  griddep_launch_dependents();  // the combine kernel waits for this grid before it reads the partial rows
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hk = blockIdx.y, split = blockIdx.z;
  const int64_t rows_all = p.n_tokens * p.group;
  const int64_t r0 = (int64_t)blockIdx.x * kRows;
  // rows run in token order, so the CTA's last row has the furthest causal limit
  const int64_t kmax = p.offset + (min(r0 + kRows, rows_all) - 1) / p.group + 1;
  int64_t lim[RPW];   // keys [0, lim) are visible to this warp's row i (0: inactive row)
  int64_t qrow[RPW];  // the row's element offset in q_ws (-1: inactive)
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int64_t R = r0 + warp * RPW + i;
    lim[i] = 0;
    qrow[i] = -1;
    if (R < rows_all) {
      const int64_t t = R / p.group;
      lim[i] = p.offset + t + 1;
      qrow[i] = (t * p.heads + hk * p.group + (R - t * p.group)) * HD;
    }
  }

  // this split's keys
  const int64_t per = (((p.cache_len + p.splits - 1) / p.splits) + kKeyTile - 1) / kKeyTile * kKeyTile;
  const int64_t kbeg = (int64_t)split * per;
  const int64_t kend = min(kbeg + per, kmax);
  const int ntiles = kend > kbeg ? (int)((kend - kbeg + kKeyTile - 1) / kKeyTile) : 0;
  const T* kc = static_cast<const T*>(p.k_cache) + hk * p.cache_sh;
  const T* vc = static_cast<const T*>(p.v_cache) + hk * p.cache_sh;
  auto issue = [&](int tile) {
    const int64_t k0 = kbeg + (int64_t)tile * kKeyTile;
    const int nv = (int)min((int64_t)kKeyTile, kend - k0);
    T* kt = reinterpret_cast<T*>(tiles + (tile & 1) * (SM::kKT + SM::kVT));
    T* vt = reinterpret_cast<T*>(tiles + (tile & 1) * (SM::kKT + SM::kVT) + SM::kKT);
    for (int i = tid; i < kKeyTile * VPR; i += kWarps * 32) {
      const int row = i / VPR, col = (i % VPR) * SM::kVec;
      const bool ok = row < nv;  // rows past the split's end are zero-filled
      const int64_t src = (k0 + (ok ? row : 0)) * HD + col;
      cp_async16((uint32_t)__cvta_generic_to_shared(kt + row * SM::kKRow + col), kc + src, ok);
      cp_async16((uint32_t)__cvta_generic_to_shared(vt + row * HD + col), vc + src, ok);
    }
  };
  const bool early = ntiles > 0 && kbeg + kKeyTile <= p.offset;  // tile 0 holds earlier calls' keys only
  if (early) issue(0);
  griddep_wait();
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    float qv[DPL];
    if (qrow[i] >= 0) {
      ld_run<T, DPL, true>(static_cast<const T*>(p.q_ws) + qrow[i] + lane * DPL, qv);
    } else {
#pragma unroll
      for (int e = 0; e < DPL; ++e) qv[e] = 0.f;
    }
    st_run<float, DPL, true>(qs + (warp * RPW + i) * HD + lane * DPL, qv);
  }
  if (ntiles > 0 && !early) issue(0);
  cp_async_commit();

  float m[RPW], lsum[RPW], o[RPW][DPL];
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    m[i] = -INFINITY;
    lsum[i] = 0.f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) o[i][e] = 0.f;
  }
  float* ps = ps_all + warp * RPW * kKeyTile;

  for (int tile = 0; tile < ntiles; ++tile) {
    if (tile + 1 < ntiles) issue(tile + 1);
    cp_async_commit();
    cp_async_wait<1>();  // this tile's copies (and the q rows' stores, by the barrier) are done
    __syncthreads();
    const int64_t k0 = kbeg + (int64_t)tile * kKeyTile;
    const int nvalid = (int)min((int64_t)kKeyTile, kend - k0);  // uniform
    const T* kt = reinterpret_cast<const T*>(tiles + (tile & 1) * (SM::kKT + SM::kVT));
    const T* vt = reinterpret_cast<const T*>(tiles + (tile & 1) * (SM::kKT + SM::kVT) + SM::kKT);
    // scores: lane = key, four partial sums per row
    float acc[RPW][4];
#pragma unroll
    for (int i = 0; i < RPW; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    const T* krow = kt + lane * SM::kKRow;
#pragma unroll 4
    for (int d = 0; d < HD; d += SM::kVec) {
      float kv[SM::kVec];
      load_vec<T>(krow + d, kv, SM::kVec);
#pragma unroll
      for (int i = 0; i < RPW; ++i) {
        const float4* q4 = reinterpret_cast<const float4*>(qs + (warp * RPW + i) * HD + d);
#pragma unroll
        for (int e = 0; e < SM::kVec; e += 4) {
          const float4 qv = q4[e / 4];
          acc[i][0] = fmaf(qv.x, kv[e], acc[i][0]);
          acc[i][1] = fmaf(qv.y, kv[e + 1], acc[i][1]);
          acc[i][2] = fmaf(qv.z, kv[e + 2], acc[i][2]);
          acc[i][3] = fmaf(qv.w, kv[e + 3], acc[i][3]);
        }
      }
    }
    // online softmax per row
    const int64_t kpos = k0 + lane;
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const bool ok = lane < nvalid && kpos < lim[i];
      const float sv = ok ? ((acc[i][0] + acc[i][1]) + (acc[i][2] + acc[i][3])) * p.scale : -INFINITY;
      float tm = sv;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, off));
      const float mn = fmaxf(m[i], tm);
      const float alpha = mn == -INFINITY ? 1.f : __expf(m[i] - mn);
      const float pj = ok ? __expf(sv - mn) : 0.f;
      lsum[i] = lsum[i] * alpha + pj;
#pragma unroll
      for (int e = 0; e < DPL; ++e) o[i][e] *= alpha;
      m[i] = mn;
      ps[i * kKeyTile + lane] = pj;
    }
    __syncwarp();
    // output: lane = features [lane * DPL, +DPL); keys past nvalid have p = 0 and zero rows
#pragma unroll 8
    for (int j = 0; j < kKeyTile; ++j) {
      float vv[DPL];
      if constexpr (DPL * sizeof(T) >= 16) {
        load_vec<T>(vt + j * HD + lane * DPL, vv, DPL);
      } else {
#pragma unroll
        for (int e = 0; e < DPL; ++e) vv[e] = to_f(vt[j * HD + lane * DPL + e]);
      }
#pragma unroll
      for (int i = 0; i < RPW; ++i) {
        const float pr = ps[i * kKeyTile + j];
#pragma unroll
        for (int e = 0; e < DPL; ++e) o[i][e] = fmaf(pr, vv[e], o[i][e]);
      }
    }
    __syncthreads();  // every warp is done with this buffer before it is refilled
  }
  cp_async_wait<0>();

  // this warp's rows: the sum over lanes, then the output or the partial row
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) lsum[i] += __shfl_xor_sync(0xffffffffu, lsum[i], off);
    if (qrow[i] < 0) continue;
    const int64_t row = qrow[i] / HD;  // t * heads + h
    const int64_t t = row / p.heads;
    const int h = (int)(row - t * p.heads);
    if (p.splits == 1) {
      const T* gate = static_cast<const T*>(p.qg) + t * p.qg_st + (int64_t)h * 2 * HD + HD;
      T* dst = static_cast<T*>(p.out) + t * p.out_st + (int64_t)h * HD;
      const float inv = 1.f / lsum[i];
#pragma unroll
      for (int e = 0; e < DPL; ++e) {
        const int d = lane * DPL + e;
        const float att = round_to<T>(o[i][e] * inv);
        const float gt = round_to<T>(sigmoid_f(to_f(gate[d])));
        dst[d] = from_f<T>(att * gt);
      }
    } else {
      float* pr = p.part + ((size_t)split * p.n_tokens * p.heads + row) * (HD + 4);
      st_run<float, DPL, true>(pr + lane * DPL, o[i]);
      if (lane == 0) {
        pr[HD] = m[i];
        pr[HD + 1] = lsum[i];
      }
    }
  }
}

// Adds the splits' partial rows: out = sum_s e^(m_s - m) o_s / sum_s e^(m_s - m) l_s.
// One CTA per (output row, 64 features), launched as a programmatic dependent
// of the attention kernel: warp w takes splits w, w + 8, ... with all of its
// loads issued at once (two features per lane), weights them by its own
// largest max, and the eight warps' sums meet in shared memory.
constexpr int kMaxSplits = 160;
constexpr int kCombWarps = 8;
constexpr int kCombFeat = 64;

template <typename T>
__global__ void __launch_bounds__(kCombWarps * 32) attn_combine_kernel(const AttnParams p) {
  constexpr int kPer = kMaxSplits / kCombWarps;
  __shared__ float wm[kCombWarps], wl[kCombWarps];
  __shared__ float2 wacc[kCombWarps][32];
  griddep_wait();
  const int hd = p.head_dim, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x;  // t * heads + h
  const int f = blockIdx.y * kCombFeat + 2 * lane;
  const bool fok = f < hd;
  const size_t stride = (size_t)p.n_tokens * p.heads * (hd + 4);
  const float* base = p.part + row * (hd + 4);
  float ms[kPer], ls[kPer];
  float2 os[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int s = warp + j * kCombWarps;
    ms[j] = -INFINITY;
    ls[j] = 0.f;
    os[j] = make_float2(0.f, 0.f);
    if (s < p.splits) {
      const float* src = base + s * stride;
      ms[j] = src[hd];
      ls[j] = src[hd + 1];
      if (fok) os[j] = *reinterpret_cast<const float2*>(src + f);
    }
  }
  float mw = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPer; ++j) mw = fmaxf(mw, ms[j]);
  float lw = 0.f, ax = 0.f, ay = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const float w = ms[j] == -INFINITY ? 0.f : __expf(ms[j] - mw);
    lw = fmaf(w, ls[j], lw);
    ax = fmaf(w, os[j].x, ax);
    ay = fmaf(w, os[j].y, ay);
  }
  if (lane == 0) {
    wm[warp] = mw;
    wl[warp] = lw;
  }
  wacc[warp][lane] = make_float2(ax, ay);
  __syncthreads();
  if (warp != 0 || !fok) return;
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kCombWarps; ++w) M = fmaxf(M, wm[w]);
  float L = 0.f, X = 0.f, Y = 0.f;
#pragma unroll
  for (int w = 0; w < kCombWarps; ++w) {
    const float c = wm[w] == -INFINITY ? 0.f : __expf(wm[w] - M);
    L = fmaf(c, wl[w], L);
    X = fmaf(c, wacc[w][lane].x, X);
    Y = fmaf(c, wacc[w][lane].y, Y);
  }
  const float inv = 1.f / L;
  const int64_t t = row / p.heads;
  const int h = (int)(row - t * p.heads);
  const T* gate = static_cast<const T*>(p.qg) + t * p.qg_st + (int64_t)h * 2 * hd + hd;
  T* dst = static_cast<T*>(p.out) + t * p.out_st + (int64_t)h * hd;
  const float a0 = round_to<T>(X * inv), a1 = round_to<T>(Y * inv);
  const float g0 = round_to<T>(sigmoid_f(to_f(gate[f]))), g1 = round_to<T>(sigmoid_f(to_f(gate[f + 1])));
  dst[f] = from_f<T>(a0 * g0);
  dst[f + 1] = from_f<T>(a1 * g1);
}

// ------------------------------------------------- prefill, tensor cores
// bf16 prefill on mma.sync m16n8k16 (bf16 x bf16 -> float32), FA2-style: one
// CTA per (128 queries, query head), eight warps of 16 query rows sharing
// each K/V tile.  K and V
// tiles of 64 keys (the key/value head of the group) pass through shared
// memory by cp.async, double-buffered; each 16-byte chunk of a row sits at
// chunk ^ (row & 7) so that ldmatrix reads are free of bank conflicts.
// S = Q K^T: A fragments of Q by ldmatrix, B fragments of K by ldmatrix (K
// rows are the B operand's columns); the online softmax runs on the S
// fragments; P goes from the S accumulators straight into A fragments;
// O += P V: B fragments of V by ldmatrix.trans.  The causal mask applies on
// the tiles that cross the diagonal.
constexpr int kMQ = 128;  // queries per CTA: eight warps of 16 rows
constexpr int kMmaThreads = 256;
constexpr int kMK = 64;   // keys per tile

template <int HD>
struct MmaSmem {
  static constexpr size_t kTile = (size_t)kMK * HD * 2;  // one K or V tile, bf16
  static constexpr size_t kQ = (size_t)kMQ * HD * 2;
  static constexpr size_t kBytes = kQ + 4 * kTile;      // Q, K[2], V[2]
};

__device__ __forceinline__ uint32_t swz(int row, int col, int hd) {
  // byte offset of element (row, col) in a [rows][hd] bf16 tile, 16-byte chunks XOR-swizzled
  return (uint32_t)(row * hd * 2 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int HD>
__global__ void __launch_bounds__(kMmaThreads, 1) attn_mma_kernel(const AttnParams p) {
  using SM = MmaSmem<HD>;
  constexpr int NT = HD / 8;      // output n-tiles of 8 features
  constexpr int KC = HD / 8;      // 16-byte chunks per row
  extern __shared__ __align__(16) unsigned char smem_mma[];
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem_mma);
  const uint32_t sQ = sbase, sK0 = sbase + SM::kQ, sV0 = sK0 + 2 * SM::kTile;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  // query tiles in reverse order: the tiles with the most keys (the last
  // queries) start first and the short ones fill the tail of the grid
  const int h = blockIdx.x, hk = h / p.group;
  const int64_t q0 = (int64_t)(gridDim.y - 1 - blockIdx.y) * kMQ;  // first query (token index of this call)
  const __nv_bfloat16* qw = static_cast<const __nv_bfloat16*>(p.q_ws);
  const __nv_bfloat16* kc = static_cast<const __nv_bfloat16*>(p.k_cache) + hk * p.cache_sh;
  const __nv_bfloat16* vc = static_cast<const __nv_bfloat16*>(p.v_cache) + hk * p.cache_sh;
  // keys this CTA needs: up to the newest of its queries
  const int64_t q_last = min(q0 + kMQ, p.n_tokens) - 1;
  const int64_t kneed = p.offset + q_last + 1;
  const int ntiles = (int)((kneed + kMK - 1) / kMK);

  // Q tile (rows past n_tokens zero-filled)
  for (int i = tid; i < kMQ * KC; i += kMmaThreads) {
    const int r = i / KC, c = (i % KC) * 8;
    const int64_t t = q0 + r;
    const bool ok = t < p.n_tokens;
    cp_async16(sQ + swz(r, c, HD), qw + ((ok ? t : 0) * p.heads + h) * HD + c, ok);
  }
  auto load_kv = [&](int tile, int buf) {
    const int64_t k0 = (int64_t)tile * kMK;
    for (int i = tid; i < kMK * KC; i += kMmaThreads) {
      const int r = i / KC, c = (i % KC) * 8;
      const int64_t kp = k0 + r;
      const bool ok = kp < kneed;
      const int64_t src = (ok ? kp : 0) * HD + c;
      cp_async16(sK0 + buf * SM::kTile + swz(r, c, HD), kc + src, ok);
      cp_async16(sV0 + buf * SM::kTile + swz(r, c, HD), vc + src, ok);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows g and g + 8 of this warp
  const float sl2 = p.scale * 1.4426950408889634f;           // scores in log2 units
  const int64_t qpos0 = p.offset + q0 + warp * 16 + g, qpos1 = qpos0 + 8;

  for (int tile = 0; tile < ntiles; ++tile) {
    const int buf = tile & 1;
    if (tile + 1 < ntiles) load_kv(tile + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();  // this tile (and Q) have landed
    __syncthreads();
    const uint32_t sK = sK0 + buf * SM::kTile, sV = sV0 + buf * SM::kTile;

    // S = Q K^T for this warp's 16 rows x 64 keys
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t a[4];
      ldsm_x4(sQ + swz(warp * 16 + (lane & 15), ks * 16 + (lane >> 4) * 8, HD), a);
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of key n-tiles
        uint32_t b[4];
        const int krow = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int kcol = ks * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(sK + swz(krow, kcol, HD), b);
        mma16816(s[2 * np], a, b[0], b[1]);
        mma16816(s[2 * np + 1], a, b[2], b[3]);
      }
    }
    // mask and online softmax (rows g: s[n][0..1], g + 8: s[n][2..3])
    const int64_t k0 = (int64_t)tile * kMK;
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t kp = k0 + n * 8 + 2 * t4 + e;
        s[n][e] = kp <= qpos0 ? s[n][e] * sl2 : -INFINITY;
        s[n][2 + e] = kp <= qpos1 ? s[n][2 + e] * sl2 : -INFINITY;
        mx0 = fmaxf(mx0, s[n][e]);
        mx1 = fmaxf(mx1, s[n][2 + e]);
      }
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float al0 = mx0 == -INFINITY ? 1.f : exp2f(m0 - mx0), al1 = mx1 == -INFINITY ? 1.f : exp2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    l0 *= al0;
    l1 *= al1;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= al0;
      o[n][1] *= al0;
      o[n][2] *= al1;
      o[n][3] *= al1;
    }
    uint32_t pa[4][4];  // P as A fragments: 4 k-steps of 16 keys
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p00 = m0 == -INFINITY ? 0.f : exp2f(s[n][0] - m0), p01 = m0 == -INFINITY ? 0.f : exp2f(s[n][1] - m0);
      const float p10 = m1 == -INFINITY ? 0.f : exp2f(s[n][2] - m1), p11 = m1 == -INFINITY ? 0.f : exp2f(s[n][3] - m1);
      l0 += p00 + p01;
      l1 += p10 + p11;
      pa[n >> 1][(n & 1) * 2] = cvt_bf16x2(p00, p01);
      pa[n >> 1][(n & 1) * 2 + 1] = cvt_bf16x2(p10, p11);
    }
    // O += P V
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {  // pairs of feature n-tiles
        uint32_t b[4];
        const int vrow = ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int vcol = np * 16 + (lane >> 4) * 8;
        ldsm_x4_t(sV + swz(vrow, vcol, HD), b);
        mma16816(o[2 * np], pa[ks], b[0], b[1]);
        mma16816(o[2 * np + 1], pa[ks], b[2], b[3]);
      }
    }
    __syncthreads();  // every warp is done with this buffer before it is refilled
  }
  cp_async_wait<0>();

  // rows g and g + 8: normalize, gate, store
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const __nv_bfloat16* qg = static_cast<const __nv_bfloat16*>(p.qg);
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int64_t t = q0 + warp * 16 + g + half * 8;
    if (t >= p.n_tokens) continue;
    const float inv = 1.f / (half ? l1 : l0);
    const __nv_bfloat16* gate = qg + t * p.qg_st + (int64_t)h * 2 * HD + HD;
    __nv_bfloat16* dst = out + t * p.out_st + (int64_t)h * HD;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int d = n * 8 + 2 * t4;
      const float a0 = round_to<__nv_bfloat16>(o[n][half * 2] * inv);
      const float a1 = round_to<__nv_bfloat16>(o[n][half * 2 + 1] * inv);
      const float g0 = round_to<__nv_bfloat16>(sigmoid_f(__bfloat162float(gate[d])));
      const float g1 = round_to<__nv_bfloat16>(sigmoid_f(__bfloat162float(gate[d + 1])));
      *reinterpret_cast<uint32_t*>(dst + d) = cvt_bf16x2(a0 * g0, a1 * g1);
    }
  }
}

// ------------------------------------------------------------------ prefill on tcgen05
// attn_tc_kernel<HD>: bf16 prefill (head_dim 128 or 256), one CTA per (128
// queries, head), keys in tiles of 64.  Warp 0 lane 0 loads Q once and the K
// and V tiles (two buffers each, with barriers of their own: a K buffer is
// refilled once S has read it, a V buffer once P V has) by TMA, zero-filled
// past the cache length; warp 1 lane 0 issues
//   S_j  = Q K_j^T   M = 128 queries, N = 64 keys, K = HD    two TMEM buffers
//   O   += P_j V_j   M = 128, N = HD, K = 64 keys            P read from TMEM, V MN-major
// (at head_dim 256, Q is copied into TMEM first and S reads it there) and
// warps 4-11 turn S_j into P_j with an online softmax in log2 units (a query
// row per TMEM lane, its 64 keys split between warps 4-7 and 8-11), P written
// as packed bf16 over the first 32 columns of S_j's buffer.  A row's O and
// running sum l are rescaled only when its maximum grows by more than
// kTcRescale (until then every p <= 2^kTcRescale); l sums the unrounded p, as
// attn_mma_kernel does.  The end: O / l through shared memory (the idle K
// buffers), then whole rows per warp for the sigmoid gate and the bf16
// rounding of attn_mma_kernel.  Every wait is bounded; a timeout is recorded
// in g_attn_error.
constexpr int kTcQ = 128, kTcK = 64, kTcThreads = 384;
constexpr float kTcRescale = 8.f;
constexpr unsigned long long kTcWaitNs = 2000000000ull;

__device__ unsigned g_attn_error = 0;

template <int HD>
struct TcSmem {
  static constexpr uint32_t kQBytes = kTcQ * HD * 2;   // HD/64 K-blocks of 128 rows x 128 B, SW128
  static constexpr uint32_t kKVBytes = kTcK * HD * 2;  // HD/64 blocks of 64 rows x 128 B, SW128
  static constexpr uint32_t OFF_Q = 0, OFF_K = kQBytes, OFF_V = OFF_K + 2 * kKVBytes;
  static constexpr size_t kBytes = 1024 + OFF_V + 2 * (size_t)kKVBytes;
};

// K and V tiles have barriers of their own: a K buffer is free once S_j has
// read it, a V buffer once O += P_j V_j has.
enum TcBar { T_Q_FULL, T_K_FULL0, T_K_FULL1, T_V_FULL0, T_V_FULL1, T_K_EMPTY0, T_K_EMPTY1, T_V_EMPTY0, T_V_EMPTY1,
             T_S_FULL0, T_S_FULL1, T_P_READY0, T_P_READY1, T_PV_DONE, T_O_FULL, T_QT_READY, T_DRAIN, T_NBARS };

__device__ __forceinline__ void tc_record_error(volatile int* abort_flag) {
  *abort_flag = 1;
  atomicOr(&g_attn_error, sm100::kErrTimeout);
}

template <int HD>
__global__ void __launch_bounds__(kTcThreads, HD == 128 ? 2 : 1) attn_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                                                              const __grid_constant__ CUtensorMap kmap,
                                                              const __grid_constant__ CUtensorMap vmap,
                                                              const AttnParams p) {
  using namespace sm100;
  using SM = TcSmem<HD>;
  constexpr int KB = HD / 64;                                   // 64-wide blocks of the head dim
  constexpr uint32_t kCols = HD + 2 * kTcK <= 256 ? 256 : 512;  // O, then the two S buffers
  // At head_dim 256, Q also lives in TMEM (its last 128 columns, bf16 pairs)
  // as the A operand of S, so that each S product reads only K from shared
  // memory.  At 128 it stays in shared memory (two CTAs share an SM's TMEM).
  constexpr bool QT = HD == 256;
  constexpr uint32_t QCOL = HD + 2 * kTcK;
  static_assert(!QT || QCOL + HD / 2 <= kCols, "Q fits the TMEM allocation");
  extern __shared__ unsigned char smem_tc[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_tc) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bars[T_NBARS];
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ float red_max[2][kTcQ];  // row maxima (then row sums) of the two softmax halves
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x, hk = h / p.group;
  // query tiles in reverse order: the tiles with the most keys start first
  const int64_t q0 = (int64_t)(gridDim.y - 1 - blockIdx.y) * kTcQ;
  const int64_t q_last = min(q0 + kTcQ, p.n_tokens) - 1;
  const int64_t kneed = p.offset + q_last + 1;
  const int ntiles = (int)((kneed + kTcK - 1) / kTcK);

  if (tid == 0) {
    abort_flag = 0;
    for (int i = 0; i < T_NBARS; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base, kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      mbar_arrive_expect_tx(&bars[T_Q_FULL], SM::kQBytes);
#pragma unroll
      for (int kb = 0; kb < KB; ++kb)
        tma_load_3d(base + SM::OFF_Q + kb * (kTcQ * 128), &qmap, &bars[T_Q_FULL], kb * 64, h, (int)q0);
      // K_i, then V_(i-1): K_i waits for S_(i-2) to have read its buffer and
      // V_(i-1) for O += P_(i-3) V_(i-3), in the order the MMAs complete.
      uint32_t kloads[2] = {0, 0}, vloads[2] = {0, 0};
      auto load = [&](int j, bool is_v) -> bool {
        const int b = j & 1;
        const int empty = (is_v ? T_V_EMPTY0 : T_K_EMPTY0) + b, full = (is_v ? T_V_FULL0 : T_K_FULL0) + b;
        if (j >= 2 && !mbar_wait(&bars[empty], (uint32_t)(((j >> 1) - 1) & 1), kTcWaitNs)) return false;
        mbar_arrive_expect_tx(&bars[full], SM::kKVBytes);
        unsigned char* dst = base + (is_v ? SM::OFF_V : SM::OFF_K) + b * SM::kKVBytes;
#pragma unroll
        for (int kb = 0; kb < KB; ++kb)
          tma_load_3d(dst + kb * (kTcK * 128), is_v ? &vmap : &kmap, &bars[full], kb * 64, j * kTcK, hk);
        ++(is_v ? vloads : kloads)[b];
        return true;
      };
      for (int i = 0; i <= ntiles && !abort_flag; ++i) {
        if ((i < ntiles && !load(i, false)) || (i >= 1 && !load(i - 1, true))) {
          tc_record_error(&abort_flag);
          break;
        }
      }
      // every copy this thread started lands before the CTA releases its memory
      mbar_wait(&bars[T_Q_FULL], 0, kTcWaitNs);
      for (int b = 0; b < 2; ++b) {
        if (kloads[b]) mbar_wait(&bars[T_K_FULL0 + b], (kloads[b] - 1) & 1, kTcWaitNs);
        if (vloads[b]) mbar_wait(&bars[T_V_FULL0 + b], (vloads[b] - 1) & 1, kTcWaitNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // S_j, then O += P_(j-1) V_(j-1): the product of tile j runs while the
    // softmax warps form P_(j-1); products from this thread run in order.
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16_f32(128, kTcK);
      const uint32_t id_o = idesc_bf16_f32_bmn(128, HD);
      const uint32_t sQ = smem_u32(base + SM::OFF_Q);
      bool ok = mbar_wait(&bars[QT ? T_QT_READY : T_Q_FULL], 0, kTcWaitNs);
      for (int j = 0; ok && j <= ntiles; ++j) {
        if (j < ntiles) {
          const int b = j & 1;
          ok = mbar_wait(&bars[T_K_FULL0 + b], (uint32_t)((j >> 1) & 1), kTcWaitNs);
          if (!ok || abort_flag) break;
          tc_fence_after();
          const uint32_t sK = smem_u32(base + SM::OFF_K + b * SM::kKVBytes);
#pragma unroll
          for (int kb = 0; kb < KB; ++kb)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              if constexpr (QT)
                mma_bf16_ts(tmem + HD + kTcK * b, tmem + QCOL + kb * 32 + ks * 8,
                            sdesc_sw128(sK + kb * (kTcK * 128) + ks * 32), id_s, kb + ks > 0);
              else
                mma_bf16(tmem + HD + kTcK * b, sdesc_sw128(sQ + kb * (kTcQ * 128) + ks * 32),
                         sdesc_sw128(sK + kb * (kTcK * 128) + ks * 32), id_s, kb + ks > 0);
            }
          mma_commit(&bars[T_S_FULL0 + b]);
          mma_commit(&bars[T_K_EMPTY0 + b]);
        }
        if (j >= 1) {
          const int jp = j - 1, bp = jp & 1;
          ok = mbar_wait_spin(&bars[T_P_READY0 + bp], (uint32_t)((jp >> 1) & 1), kTcWaitNs) &&
               mbar_wait_spin(&bars[T_V_FULL0 + bp], (uint32_t)((jp >> 1) & 1), kTcWaitNs);
          if (!ok || abort_flag) break;
          tc_fence_after();
          const uint32_t sV = smem_u32(base + SM::OFF_V + bp * SM::kKVBytes);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            mma_bf16_ts(tmem, tmem + HD + kTcK * bp + 8 * ks, sdesc_sw128_mn(sV + ks * 2048, kTcK * 128, 1024), id_o,
                        jp > 0 || ks > 0);
          mma_commit(&bars[T_PV_DONE]);
          mma_commit(&bars[T_V_EMPTY0 + bp]);
          if (j == ntiles) mma_commit(&bars[T_O_FULL]);  // O complete
        }
      }
      if (!ok) tc_record_error(&abort_flag);
      mma_commit(&bars[T_DRAIN]);
      mbar_wait(&bars[T_DRAIN], 0, kTcWaitNs);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------- softmax and output
    // Warps 4-7 take columns 0-31 of each S tile, warps 8-11 columns 32-63,
    // of the same rows (a warp's TMEM lane quarter is warp % 4).  The two
    // halves swap their row maxima through shared memory, keep partial row
    // sums, and each rescales and finally writes half of the O columns.
    const int half = (warp - 4) >> 2;
    const int q = warp & 3;                             // TMEM lane quarter
    const int r = q * 32 + lane;                        // query row of the tile
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    const int64_t qpos = p.offset + q0 + r;             // its position in the sequence
    const int64_t qpos_min = p.offset + q0;             // row 0's: no key of a half tile past it is masked
    const float sl2 = p.scale * 1.4426950408889634f;    // scores in log2 units
    constexpr int OC = HD / 2;                          // O columns of each half
    float m = -INFINITY, l0 = 0.f, l1 = 0.f;
    bool ok = true;
    if constexpr (QT) {
      // Q rows into TMEM: this half's two 64-wide K-blocks of row r, read
      // from the SW128 TMA tile (16-byte chunk c of row r at c ^ (r & 7)).
      ok = mbar_wait(&bars[T_Q_FULL], 0, kTcWaitNs);
      if (!ok) tc_record_error(&abort_flag);
      __syncwarp();
#pragma unroll 1
      for (int kbh = 0; kbh < 2; ++kbh) {
        const int kb = half * 2 + kbh;
        const unsigned char* row = base + SM::OFF_Q + kb * (kTcQ * 128) + r * 128;
        float w[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 u = *reinterpret_cast<const uint4*>(row + ((c ^ (r & 7)) * 16));
          w[4 * c] = __uint_as_float(u.x);
          w[4 * c + 1] = __uint_as_float(u.y);
          w[4 * c + 2] = __uint_as_float(u.z);
          w[4 * c + 3] = __uint_as_float(u.w);
        }
        __syncwarp();
        tmem_st32(tq + QCOL + kb * 32, w);
      }
      tmem_wait_st();
      tc_fence_before();
      named_sync(1, 256);
      if (half == 0 && r == 0) mbar_arrive(&bars[T_QT_READY]);
    }
    for (int j = 0; j < ntiles; ++j) {
      const int b = j & 1;
      ok = mbar_wait(&bars[T_S_FULL0 + b], (uint32_t)((j >> 1) & 1), kTcWaitNs);
      if (!ok) tc_record_error(&abort_flag);
      __syncwarp();
      tc_fence_after();
      float s[32];
      tmem_ld32(tq + HD + kTcK * b + 32 * half, s);
      tmem_wait_ld();
      const int64_t k0 = (int64_t)j * kTcK + 32 * half;
      const bool masked = k0 + 31 > qpos_min;  // uniform over the CTA
      // keys k0 + i with i <= lim are visible to this row
      const int64_t dpos = qpos - k0;
      const int lim = !masked ? 31 : dpos < -1 ? -1 : dpos > 31 ? 31 : (int)dpos;
      float mraw = -INFINITY;
      if (masked) {
#pragma unroll
        for (int i = 0; i < 32; ++i) mraw = i <= lim ? fmaxf(mraw, s[i]) : mraw;
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) mraw = fmaxf(mraw, s[i]);
      }
      red_max[half][r] = mraw * sl2;
      if (named_sync_or(1, 256, !ok || abort_flag)) break;  // the maxima of both halves are in
      const float mx = fmaxf(red_max[0][r], red_max[1][r]);
      // A row rescales when its maximum grows past the bound (the first
      // valid keys only set it).  The TMEM accesses are warp-collective, so
      // the whole warp takes the rescale when any of its rows needs one; the
      // other rows scale by 1.
      const bool grow = mx > m + kTcRescale;
      const bool scale_o = grow && m != -INFINITY;  // O holds products of earlier tiles
      if (__any_sync(0xffffffffu, scale_o)) {
        if (!__all_sync(0xffffffffu, mbar_wait(&bars[T_PV_DONE], (uint32_t)((j - 1) & 1), kTcWaitNs))) {
          tc_record_error(&abort_flag);  // O is left alone; the CTA is aborting
        } else {
          tc_fence_after();
          const float a = scale_o ? exp2f(m - mx) : 1.f;
#pragma unroll 1
          for (int c = half * OC; c < half * OC + OC; c += 32) {
            float o[32];
            tmem_ld32(tq + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= a;
            tmem_st32(tq + c, o);
          }
          tmem_wait_st();
          l0 *= a;
          l1 *= a;
        }
      }
      if (grow) m = mx;
      // p = 2^(s·scale·log2 e − m); m is finite here (every row sees key 0
      // in the first tile)
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        float p0 = exp2f(fmaf(s[i], sl2, -m));
        float p1 = exp2f(fmaf(s[i + 1], sl2, -m));
        if (masked) {
          p0 = i <= lim ? p0 : 0.f;
          p1 = i + 1 <= lim ? p1 : 0.f;
        }
        l0 += p0;
        l1 += p1;
        pk[i >> 1] = cvt_bf16x2(p0, p1);
      }
      // P over the first 32 columns of the S buffer: this half's 32 keys
      // packed in 16 (both halves' S reads finished before the barrier above)
      tmem_st16(tq + HD + kTcK * b + 16 * half, pk);
      tmem_wait_st();
      tc_fence_before();
      named_sync(1, 256);
      if (half == 0 && r == 0) mbar_arrive(&bars[T_P_READY0 + b]);
    }
    // O / l, gated: out = bf16(bf16(O / l) * bf16(sigmoid(gate))).  O is
    // complete on a barrier of its own: the last two products of O may both
    // be pending here (the product of the second-last tile is issued after
    // S of the last), so a parity wait on PV_DONE could pass a phase early.
    ok = ok && !abort_flag && mbar_wait(&bars[T_O_FULL], 0, kTcWaitNs);
    if (!ok && !abort_flag) tc_record_error(&abort_flag);
    red_max[half][r] = l0 + l1;
    // O / l rounded to bf16 goes through shared memory (the K buffers, idle
    // once the last S product is done): every lane reads its O columns (the
    // loads are warp-collective) and writes them into its row, 16-byte chunk
    // c of row r at chunk c ^ (r & 7); then each warp takes whole rows, so
    // that the gate loads and the output stores are contiguous runs.
    if (!named_sync_or(1, 256, !ok)) {
      __syncwarp();
      tc_fence_after();
      const float inv = 1.f / (red_max[0][r] + red_max[1][r]);
      unsigned char* stage = base + SM::OFF_K;  // kTcQ rows of HD bf16
      static_assert(2 * SM::kKVBytes >= (uint32_t)kTcQ * HD * 2, "the O tile fits the two K buffers");
      constexpr int CPR = HD / 8;               // 16-byte chunks per row
#pragma unroll 1
      for (int c = half * OC; c < half * OC + OC; c += 32) {
        float o[32];
        __syncwarp();
        tmem_ld32(tq + c, o);
        tmem_wait_ld();
#pragma unroll
        for (int d8 = 0; d8 < 32; d8 += 8) {
          uint32_t ow[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) ow[u] = cvt_bf16x2(o[d8 + 2 * u] * inv, o[d8 + 2 * u + 1] * inv);
          const int chunk = ((c + d8) >> 3) ^ (r & 7);
          *reinterpret_cast<uint4*>(stage + (size_t)r * HD * 2 + chunk * 16) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        }
      }
      named_sync(1, 256);
      // out = bf16(a * bf16(sigmoid(gate))), a = bf16(O / l); sigmoid from
      // the approximate exp2 and divide (relative error ~1e-6, well below
      // the bf16 rounding of the result)
      constexpr int RPI = 32 / CPR;  // rows per warp per step
      const int sw = warp - 4, rl = lane / CPR, cl = lane % CPR;
#pragma unroll 1
      for (int r0 = sw * RPI; r0 < kTcQ; r0 += 8 * RPI) {
        const int rr = r0 + rl;
        const int64_t t = q0 + rr;
        if (t >= p.n_tokens) continue;  // rows past the last token of a ragged tile
        const uint4 au = *reinterpret_cast<const uint4*>(stage + (size_t)rr * HD * 2 + ((cl ^ (rr & 7)) * 16));
        const uint4 gu = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.qg) + t * p.qg_st +
                                                         (int64_t)h * 2 * HD + HD + cl * 8);
        const uint32_t aw[4] = {au.x, au.y, au.z, au.w}, gw[4] = {gu.x, gu.y, gu.z, gu.w};
        uint32_t ow[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float g0 = round_to<__nv_bfloat16>(
              __fdividef(1.f, 1.f + ex2_approx(sm100::bf16_lo_f(gw[u]) * -1.4426950408889634f)));
          const float g1 = round_to<__nv_bfloat16>(
              __fdividef(1.f, 1.f + ex2_approx(sm100::bf16_hi_f(gw[u]) * -1.4426950408889634f)));
          ow[u] = cvt_bf16x2(sm100::bf16_lo_f(aw[u]) * g0, sm100::bf16_hi_f(aw[u]) * g1);
        }
        *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + t * p.out_st + (int64_t)h * HD + cl * 8) =
            make_uint4(ow[0], ow[1], ow[2], ow[3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kCols);
}

PFN_cuTensorMapEncodeTiled_v12000 attn_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

// 3-D bf16 map with 128-byte swizzle over dims {d0 (contiguous), d1, d2}
// with byte strides {s1, s2}; box {64, b1, b2}.
bool attn_map(CUtensorMap* map, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2,
              uint32_t b1, uint32_t b2) {
  auto enc = attn_map_encoder();
  if (!enc) return false;
  std::memset(map, 0, sizeof(*map));
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {64, b1, b2};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The tcgen05 prefill: Q from the prepared queries [n_tokens, heads, HD]; K
// and V from the caches [kv_heads, capacity, HD], their key extent the cache
// length (keys past it read as zeros).  False when the maps cannot be made
// (the caller then takes attn_mma_kernel).
template <int HD>
bool launch_tc(const AttnParams& p, cudaStream_t s, gdn_status* st) {
  if ((reinterpret_cast<uintptr_t>(p.qg) & 15u) || p.qg_st % 8 || (reinterpret_cast<uintptr_t>(p.out) & 15u) ||
      p.out_st % 8)
    return false;  // the output stage moves 16-byte runs of the gate and the output
  CUtensorMap qmap, kmap, vmap;
  if (!attn_map(&qmap, p.q_ws, HD, (uint64_t)p.heads, (uint64_t)p.n_tokens, (uint64_t)HD * 2,
                (uint64_t)p.heads * HD * 2, 1, kTcQ) ||
      !attn_map(&kmap, p.k_cache, HD, (uint64_t)p.cache_len, (uint64_t)p.kv_heads, (uint64_t)HD * 2,
                (uint64_t)p.cache_sh * 2, kTcK, 1) ||
      !attn_map(&vmap, p.v_cache, HD, (uint64_t)p.cache_len, (uint64_t)p.kv_heads, (uint64_t)HD * 2,
                (uint64_t)p.cache_sh * 2, kTcK, 1))
    return false;
  static DeviceFlags attr;
  constexpr size_t smem = TcSmem<HD>::kBytes;
  if (ensure_smem_attr(attn_tc_kernel<HD>, smem, attr) != cudaSuccess) {
    *st = set_error(GDN_ECUDA, "attention: shared-memory attribute");
    return true;
  }
  const int64_t qtiles = (p.n_tokens + kTcQ - 1) / kTcQ;
  if (qtiles > 65535) {
    *st = set_error(GDN_EUNSUPPORTED, "attention: at most %d tokens per call", 65535 * kTcQ);
    return true;
  }
  attn_tc_kernel<HD><<<dim3((unsigned)p.heads, (unsigned)qtiles), kTcThreads, smem, s>>>(qmap, kmap, vmap, p);
  *st = GDN_OK;
  return true;
}

template <int HD>
gdn_status launch_mma(const AttnParams& p, cudaStream_t s) {
  static DeviceFlags attr;
  constexpr size_t smem = MmaSmem<HD>::kBytes;
  if (ensure_smem_attr(attn_mma_kernel<HD>, smem, attr) != cudaSuccess)
    return set_error(GDN_ECUDA, "attention: shared-memory attribute");
  const int64_t qtiles = (p.n_tokens + kMQ - 1) / kMQ;
  if (qtiles > 65535) return set_error(GDN_EUNSUPPORTED, "attention: at most %d tokens per call", 65535 * kMQ);
  const dim3 grid((unsigned)p.heads, (unsigned)qtiles);
  attn_mma_kernel<HD><<<grid, kMmaThreads, smem, s>>>(p);
  return GDN_OK;
}

template <typename T, int HD>
void launch_prep(const AttnParams& p, bool vec, dim3 grid, cudaStream_t s) {
  const int rows = p.heads + 2 * p.kv_heads;
  if (p.n_tokens < 2 * (int64_t)sm_count()) {  // few tokens: a warp per row
    const int threads = 32 * (rows < kPrepMaxWarps ? rows : kPrepMaxWarps);
    if (vec)
      attn_prep_kernel<T, HD, true, 1><<<grid, threads, 0, s>>>(p);
    else
      attn_prep_kernel<T, HD, false, 1><<<grid, threads, 0, s>>>(p);
  } else {  // prefill: four rows per warp, at most eight warps
    const int warps = (rows + 3) / 4;
    const int threads = 32 * (warps < 8 ? warps : 8);
    if (vec)
      attn_prep_kernel<T, HD, true, 4><<<grid, threads, 0, s>>>(p);
    else
      attn_prep_kernel<T, HD, false, 4><<<grid, threads, 0, s>>>(p);
  }
}

template <typename T>
void launch_prep_hd(const AttnParams& p, bool vec, dim3 grid, cudaStream_t s) {
  switch (p.head_dim) {
    case 32: return launch_prep<T, 32>(p, vec, grid, s);
    case 64: return launch_prep<T, 64>(p, vec, grid, s);
    case 128: return launch_prep<T, 128>(p, vec, grid, s);
    default: return launch_prep<T, 256>(p, vec, grid, s);
  }
}

template <typename T>
gdn_status launch_combine(const AttnParams& p, cudaStream_t s) {
  const dim3 grid((unsigned)(p.n_tokens * p.heads), (unsigned)((p.head_dim + kCombFeat - 1) / kCombFeat));
  const cudaError_t e = launch_dependent(attn_combine_kernel<T>, grid, dim3(kCombWarps * 32), 0, s, p);
  if (e != cudaSuccess) return set_error(GDN_ECUDA, "attention combine launch: %s", cudaGetErrorString(e));
  return GDN_OK;
}

// ----------------------------------------------- decode, tensor cores
// bf16 calls with one token whose query heads of a key/value head fit 16
// rows (decode): the query rows (zero-padded to 16) times each key split on
// mma.sync m16n8k16, one warp per 32-key split tile with the operand layouts
// of attn_mma_kernel (Q by ldmatrix, K by ldmatrix, P from the score
// accumulators, V by ldmatrix.trans), an online softmax over the split's
// tiles, and the split's partial (max in natural-log units, sum, output)
// rows for attn_combine_kernel.  Each warp owns a single-buffered K/V tile;
// the first, when it holds keys cached by earlier calls only, is requested
// before the wait for the prep kernel.
constexpr int kDQ = 16;     // query rows of the MMA tile
constexpr int kDK = 32;     // keys per tile
constexpr int kDWarps = 1;  // warps (splits) per CTA: the split tiles spread over every SM

template <int HD>
struct DecSmem {
  static constexpr size_t kQ = (size_t)kDQ * HD * 2;
  static constexpr size_t kTile = (size_t)kDK * HD * 2;
  static constexpr size_t kBytes = kQ + (size_t)kDWarps * 2 * kTile;  // Q, then K and V per warp
};

template <int HD>
__global__ void __launch_bounds__(kDWarps * 32) attn_dec_mma_kernel(const AttnParams p) {
  using SM = DecSmem<HD>;
  constexpr int NT = HD / 8;  // output n-tiles of 8 features
  constexpr int KC = HD / 8;  // 16-byte chunks per row
  extern __shared__ __align__(16) unsigned char smem_dec[];
  griddep_launch_dependents();  // the combine kernel waits for this grid before it reads the partial rows
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem_dec);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int hk = blockIdx.y;
  const int split = blockIdx.x * kDWarps + warp;
  const bool live = split < p.splits;  // warp-uniform
  const uint32_t sQ = sbase, sK = sbase + (uint32_t)(SM::kQ + (size_t)warp * 2 * SM::kTile), sV = sK + SM::kTile;
  const __nv_bfloat16* kc = static_cast<const __nv_bfloat16*>(p.k_cache) + hk * p.cache_sh;
  const __nv_bfloat16* vc = static_cast<const __nv_bfloat16*>(p.v_cache) + hk * p.cache_sh;

  // this split's keys (one token: all cached keys are visible)
  const int64_t per = (((p.cache_len + p.splits - 1) / p.splits) + kKeyTile - 1) / kKeyTile * kKeyTile;
  const int64_t kbeg = (int64_t)split * per;
  const int64_t kend = live ? min(kbeg + per, p.cache_len) : kbeg;
  const int ntiles = kend > kbeg ? (int)((kend - kbeg + kDK - 1) / kDK) : 0;
  auto load_tile = [&](int tile) {  // by this warp only; rows past the split's end zero-filled
    const int64_t k0 = kbeg + (int64_t)tile * kDK;
    for (int i = lane; i < kDK * KC; i += 32) {
      const int r = i / KC, c = (i % KC) * 8;
      const int64_t kp = k0 + r;
      const bool ok = kp < kend;
      const int64_t src = (ok ? kp : k0) * HD + c;
      cp_async16(sK + swz(r, c, HD), kc + src, ok);
      cp_async16(sV + swz(r, c, HD), vc + src, ok);
    }
  };
  const bool early = ntiles > 0 && kbeg + kDK <= p.offset;  // tile 0 holds earlier calls' keys only
  if (early) load_tile(0);
  griddep_wait();
  // Q: rows r < group are the query heads hk * group + r of the token
  const __nv_bfloat16* qw = static_cast<const __nv_bfloat16*>(p.q_ws);
  for (int i = tid; i < kDQ * KC; i += kDWarps * 32) {
    const int r = i / KC, c = (i % KC) * 8;
    const bool ok = r < p.group;
    cp_async16(sQ + swz(r, c, HD), qw + (int64_t)(hk * p.group + (ok ? r : 0)) * HD + c, ok);
  }
  if (ntiles > 0 && !early) load_tile(0);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();  // Q from every thread; each warp's own tile

  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows g and g + 8
  const float sl2 = p.scale * 1.4426950408889634f;           // scores in log2 units
  for (int tile = 0; tile < ntiles; ++tile) {
    if (tile > 0) {  // single buffer: the previous tile is done (warp-synchronous ldmatrix reads)
      __syncwarp();
      load_tile(tile);
      cp_async_commit();
      cp_async_wait<0>();
      __syncwarp();
    }
    // S = Q K^T: 16 rows x 32 keys
    float s[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t a[4];
      ldsm_x4(sQ + swz(lane & 15, ks * 16 + (lane >> 4) * 8, HD), a);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t b[4];
        const int krow = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int kcol = ks * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(sK + swz(krow, kcol, HD), b);
        mma16816(s[2 * np], a, b[0], b[1]);
        mma16816(s[2 * np + 1], a, b[2], b[3]);
      }
    }
    const int64_t k0 = kbeg + (int64_t)tile * kDK;
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int n = 0; n < 4; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool ok = k0 + n * 8 + 2 * t4 + e < kend;
        s[n][e] = ok ? s[n][e] * sl2 : -INFINITY;
        s[n][2 + e] = ok ? s[n][2 + e] * sl2 : -INFINITY;
        mx0 = fmaxf(mx0, s[n][e]);
        mx1 = fmaxf(mx1, s[n][2 + e]);
      }
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float al0 = mx0 == -INFINITY ? 1.f : exp2f(m0 - mx0), al1 = mx1 == -INFINITY ? 1.f : exp2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    l0 *= al0;
    l1 *= al1;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= al0;
      o[n][1] *= al0;
      o[n][2] *= al1;
      o[n][3] *= al1;
    }
    uint32_t pa[2][4];  // P as A fragments: 2 k-steps of 16 keys
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const float p00 = m0 == -INFINITY ? 0.f : exp2f(s[n][0] - m0), p01 = m0 == -INFINITY ? 0.f : exp2f(s[n][1] - m0);
      const float p10 = m1 == -INFINITY ? 0.f : exp2f(s[n][2] - m1), p11 = m1 == -INFINITY ? 0.f : exp2f(s[n][3] - m1);
      l0 += p00 + p01;
      l1 += p10 + p11;
      pa[n >> 1][(n & 1) * 2] = cvt_bf16x2(p00, p01);
      pa[n >> 1][(n & 1) * 2 + 1] = cvt_bf16x2(p10, p11);
    }
    // O += P V
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t b[4];
        const int vrow = ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int vcol = np * 16 + (lane >> 4) * 8;
        ldsm_x4_t(sV + swz(vrow, vcol, HD), b);
        mma16816(o[2 * np], pa[ks], b[0], b[1]);
        mma16816(o[2 * np + 1], pa[ks], b[2], b[3]);
      }
    }
  }
  if (!live) return;  // no barrier follows
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  // partial rows g and g + 8 (when they are query heads): output, max (natural log), sum
  const float ln2 = 0.6931471805599453f;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = g + 8 * half;
    if (r >= p.group) continue;
    float* pr = p.part + ((size_t)split * p.n_tokens * p.heads + (size_t)(hk * p.group + r)) * (HD + 4);
#pragma unroll
    for (int n = 0; n < NT; ++n)
      *reinterpret_cast<float2*>(pr + n * 8 + 2 * t4) = make_float2(o[n][2 * half], o[n][2 * half + 1]);
    if (t4 == 0) {
      const float mm = half ? m1 : m0;
      pr[HD] = mm == -INFINITY ? -INFINITY : mm * ln2;
      pr[HD + 1] = half ? l1 : l0;
    }
  }
}

template <int HD>
gdn_status launch_dec_mma(const AttnParams& p, cudaStream_t s) {
  static DeviceFlags attr;
  constexpr size_t smem = DecSmem<HD>::kBytes;
  if (ensure_smem_attr(attn_dec_mma_kernel<HD>, smem, attr) != cudaSuccess)
    return set_error(GDN_ECUDA, "attention: shared-memory attribute");
  const dim3 grid((unsigned)((p.splits + kDWarps - 1) / kDWarps), (unsigned)p.kv_heads);
  const cudaError_t e = launch_dependent(attn_dec_mma_kernel<HD>, grid, dim3(kDWarps * 32), smem, s, p);
  if (e != cudaSuccess) return set_error(GDN_ECUDA, "attention launch: %s", cudaGetErrorString(e));
  return GDN_OK;
}

template <typename T, int HD>
gdn_status launch_fwd(const AttnParams& p, dim3 grid, cudaStream_t s) {
  static DeviceFlags attr;
  constexpr size_t smem = AttnSmem<T, HD>::kBytes;
  if (ensure_smem_attr(attn_fwd_kernel<T, HD>, smem, attr) != cudaSuccess)
    return set_error(GDN_ECUDA, "attention: shared-memory attribute");
  const cudaError_t e = launch_dependent(attn_fwd_kernel<T, HD>, grid, dim3(kWarps * 32), smem, s, p);
  if (e != cudaSuccess) return set_error(GDN_ECUDA, "attention launch: %s", cudaGetErrorString(e));
  return GDN_OK;
}

template <typename T>
gdn_status launch_fwd_hd(const AttnParams& p, dim3 grid, cudaStream_t s) {
  switch (p.head_dim) {
    case 32: return launch_fwd<T, 32>(p, grid, s);
    case 64: return launch_fwd<T, 64>(p, grid, s);
    case 128: return launch_fwd<T, 128>(p, grid, s);
    default: return launch_fwd<T, 256>(p, grid, s);
  }
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// Checks the arguments and fills everything but the workspace pointers.
gdn_status attn_setup(const gdn_attn_args* a, AttnParams* p, size_t* ws_bytes) {
  if (!a) return set_error(GDN_EINVAL, "args is NULL");
  if (a->n_tokens < 0 || a->cache_len < a->n_tokens || a->capacity < a->cache_len)
    return set_error(GDN_EINVAL, "attention needs 0 <= n_tokens <= cache_len <= capacity");
  if (a->heads <= 0 || a->kv_heads <= 0 || a->heads % a->kv_heads)
    return set_error(GDN_EINVAL, "heads must be a positive multiple of kv_heads");
  if (a->head_dim != 32 && a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256)
    return set_error(GDN_EUNSUPPORTED, "head_dim must be 32, 64, 128 or 256 (got %d)", a->head_dim);
  if (a->rotary_dim < 0 || a->rotary_dim > a->head_dim || a->rotary_dim % 2)
    return set_error(GDN_EINVAL, "rotary_dim must be even and at most head_dim");
  if (a->act_dtype != GDN_F32 && a->act_dtype != GDN_BF16)
    return set_error(GDN_EUNSUPPORTED, "attention runs float32 or bf16 activations");
  if (a->n_tokens > 0 && (!a->qg || !a->k_new || !a->v_new || !a->q_norm || !a->k_norm || !a->k_cache ||
                          !a->v_cache || !a->out))
    return set_error(GDN_EINVAL, "tensor pointers must be non-NULL");
  const size_t es = a->act_dtype == GDN_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(a->k_cache) | reinterpret_cast<uintptr_t>(a->v_cache)) & 15u)
    return set_error(GDN_EINVAL, "the caches must be 16-byte aligned");
  if (a->n_tokens > 0x7fffffffLL || a->cache_len > 0x7fffffffLL)
    return set_error(GDN_EUNSUPPORTED, "n_tokens and cache_len must be < 2^31");
  p->n_tokens = a->n_tokens;
  p->cache_len = a->cache_len;
  p->offset = a->cache_len - a->n_tokens;
  p->heads = a->heads;
  p->kv_heads = a->kv_heads;
  p->head_dim = a->head_dim;
  p->rotary_dim = a->rotary_dim;
  p->group = a->heads / a->kv_heads;
  p->eps = a->eps;
  p->scale = a->scale;
  for (int i = 0; i < a->rotary_dim / 2; ++i)
    p->inv_freq[i] = std::exp(-2.0 * i / a->rotary_dim * std::log((double)a->rope_base));
  p->qg = a->qg;
  p->qg_st = a->qg_stride_t;
  p->k_new = a->k_new;
  p->k_st = a->k_stride_t;
  p->v_new = a->v_new;
  p->v_st = a->v_stride_t;
  p->q_norm = a->q_norm;
  p->k_norm = a->k_norm;
  p->k_cache = a->k_cache;
  p->v_cache = a->v_cache;
  p->cache_sh = a->capacity * a->head_dim;
  p->out = a->out;
  p->out_st = a->out_stride_t;
  // key splits: enough CTAs for the machine when the rows are few (decode)
  const int64_t row_ctas = (a->n_tokens * p->group + kRows - 1) / kRows * a->kv_heads;
  int64_t splits = 1;
  if (row_ctas > 0 && row_ctas < 2 * 148) {
    splits = (2 * 148 + row_ctas - 1) / row_ctas;
    const int64_t max_by_keys = (a->cache_len + kKeyTile - 1) / kKeyTile;  // one tile a split at least
    if (splits > max_by_keys) splits = max_by_keys;
    if (splits > kMaxSplits) splits = kMaxSplits;
    if (splits < 1) splits = 1;
  }
  // bf16 prefill with head_dim >= 64 runs the tensor-core kernel, one key split
  if (a->act_dtype == GDN_BF16 && a->head_dim >= 64 && (a->n_tokens >= kMQ || splits == 1)) splits = 1;
  p->splits = (int)splits;
  const size_t q_bytes = align256((size_t)a->n_tokens * a->heads * a->head_dim * es);
  const size_t part_bytes =
      splits > 1 ? align256((size_t)splits * a->n_tokens * a->heads * (a->head_dim + 4) * 4) : 0;
  *ws_bytes = q_bytes + part_bytes;
  return GDN_OK;
}

}  // namespace

cudaError_t read_and_clear_attn_error(unsigned* code) {
  cudaError_t e = cudaMemcpyFromSymbol(code, g_attn_error, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  if (*code) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_attn_error, &zero, sizeof(unsigned));
  }
  return e;
}
}  // namespace gdn

extern "C" gdn_status gdn_attention_workspace_size(const gdn_attn_args* a, size_t* bytes) {
  gdn::AttnParams p;
  if (!bytes) return gdn::set_error(GDN_EINVAL, "bytes is NULL");
  return gdn::attn_setup(a, &p, bytes);
}

extern "C" gdn_status gdn_attention(const gdn_attn_args* a, gdn_stream_t stream) {
  gdn::AttnParams p;
  size_t need = 0;
  gdn_status st = gdn::attn_setup(a, &p, &need);
  if (st != GDN_OK) return st;
  if (a->n_tokens == 0) return GDN_OK;
  if (!a->workspace || a->workspace_bytes < need)
    return gdn::set_error(GDN_EINVAL, "workspace too small: %zu bytes needed", need);
  if (reinterpret_cast<uintptr_t>(a->workspace) & 15u) return gdn::set_error(GDN_EINVAL, "the workspace must be 16-byte aligned");
  const size_t es = a->act_dtype == GDN_F32 ? 4 : 2;
  unsigned char* ws = static_cast<unsigned char*>(a->workspace);
  p.q_ws = ws;
  p.part = reinterpret_cast<float*>(ws + gdn::align256((size_t)a->n_tokens * a->heads * a->head_dim * es));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // vector accesses in the prep kernel when every row start is aligned to a lane's run of features
  const size_t run = (size_t)(a->head_dim / 32) * es, run_t = run < 16 ? run : 16;
  const size_t run_f = (size_t)(a->head_dim / 32) * 4 < 16 ? (size_t)(a->head_dim / 32) * 4 : 16;
  auto al = [](const void* ptr, size_t n) { return reinterpret_cast<uintptr_t>(ptr) % n == 0; };
  const bool vec = al(a->qg, run_t) && al(a->k_new, run_t) && al(a->v_new, run_t) &&
                   (a->qg_stride_t * (int64_t)es) % (int64_t)run_t == 0 &&
                   (a->k_stride_t * (int64_t)es) % (int64_t)run_t == 0 &&
                   (a->v_stride_t * (int64_t)es) % (int64_t)run_t == 0 && al(a->q_norm, run_f) && al(a->k_norm, run_f);
  const dim3 pgrid((unsigned)a->n_tokens);  // one CTA per token
  const int64_t row_blocks = (a->n_tokens * p.group + gdn::kRows - 1) / gdn::kRows;
  if (row_blocks > 0x7fffffffLL) return gdn::set_error(GDN_EUNSUPPORTED, "too many rows for one call");
  const dim3 fgrid((unsigned)row_blocks, (unsigned)a->kv_heads, (unsigned)p.splits);
  if (a->act_dtype == GDN_F32) {
    gdn::launch_prep_hd<float>(p, vec, pgrid, s);
    st = gdn::launch_fwd_hd<float>(p, fgrid, s);
    if (st == GDN_OK && p.splits > 1) st = gdn::launch_combine<float>(p, s);
  } else {
    // a plain launch: the attention kernel, its dependent, reads keys cached
    // by earlier calls before it waits, which is safe only when everything
    // before the prep kernel has completed once it starts
    gdn::launch_prep_hd<__nv_bfloat16>(p, vec, pgrid, s);
    if (p.splits == 1 && a->head_dim >= 64) {  // prefill: the tensor-core kernel
      switch (a->head_dim) {
        case 64: st = gdn::launch_mma<64>(p, s); break;
        case 128:
          if (!gdn::launch_tc<128>(p, s, &st)) st = gdn::launch_mma<128>(p, s);
          break;
        default:
          if (!gdn::launch_tc<256>(p, s, &st)) st = gdn::launch_mma<256>(p, s);
          break;
      }
    } else if (a->n_tokens == 1 && p.group <= gdn::kDQ && a->head_dim >= 64) {  // decode: tensor cores
      switch (a->head_dim) {
        case 64: st = gdn::launch_dec_mma<64>(p, s); break;
        case 128: st = gdn::launch_dec_mma<128>(p, s); break;
        default: st = gdn::launch_dec_mma<256>(p, s); break;
      }
    } else {
      st = gdn::launch_fwd_hd<__nv_bfloat16>(p, fgrid, s);
    }
    if (st == GDN_OK && p.splits > 1) st = gdn::launch_combine<__nv_bfloat16>(p, s);
  }
  if (st != GDN_OK) return st;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return gdn::set_error(GDN_ECUDA, "attention launch: %s", cudaGetErrorString(e));
  return GDN_OK;
}
