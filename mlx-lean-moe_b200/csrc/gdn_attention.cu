// The softmax-attention layer's core (the reference's Qwen3_5Attention
// between its projections, qw/attention.py:56-96, with the GrowingKVCache of
// cache/kv_cache.py): q/k RMS norms with weights, rotary embedding of the
// leading rotary_dim features (model/rope.py: feature i pairs with
// i + rotary_dim / 2, angle = position * base^(-2i / rotary_dim)), the append
// of this call's keys and values to a head-major cache, grouped-query
// attention with the causal mask aligned to the newest query, and the
// output gate sigmoid(gate) carried in q_proj's second half.
//
// attn_prep_kernel     one warp per (token, row of q / k / v heads): the
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
// attn_mma_kernel      bf16 prefill (calls with enough rows for one key
//                      split) on the tensor cores: see its comment below.
#include <cuda_bf16.h>

#include <cmath>
#include <cstring>

#include "gdn_api.h"
#include "gdn_common.cuh"

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
// One warp per (token, head row): rows [0, heads) are queries, then the
// kv_heads keys, then the kv_heads values; each lane holds head_dim / 32
// consecutive features.  The norm reduces by shuffles; the rotation reads its
// partner features from the warp's row in shared memory.
constexpr int kPrepWarps = 8;

template <typename T>
__device__ __forceinline__ void load_feat(const T* src, float (&x)[8], int dpl) {
  for (int e = 0; e < dpl; ++e) x[e] = to_f(src[e]);
}

template <typename T>
__global__ void __launch_bounds__(kPrepWarps * 32) attn_prep_kernel(const AttnParams p) {
  __shared__ float xs[kPrepWarps][kMaxHeadDim];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = p.heads + 2 * p.kv_heads;
  const int64_t item = (int64_t)blockIdx.x * kPrepWarps + warp;
  if (item >= p.n_tokens * rows) return;  // the whole warp
  const int64_t t = item / rows;
  const int row = (int)(item % rows);
  const int hd = p.head_dim, dpl = hd / 32, d0 = lane * dpl;
  const bool is_q = row < p.heads, is_k = !is_q && row < p.heads + p.kv_heads;
  const int h = is_q ? row : is_k ? row - p.heads : row - p.heads - p.kv_heads;
  const int64_t pos = p.offset + t;
  if (!is_q && !is_k) {  // v: a copy into the cache
    const T* src = static_cast<const T*>(p.v_new) + t * p.v_st + (int64_t)h * hd + d0;
    T* dst = static_cast<T*>(p.v_cache) + h * p.cache_sh + pos * hd + d0;
    for (int e = 0; e < dpl; ++e) dst[e] = src[e];
    return;
  }
  const T* src = is_q ? static_cast<const T*>(p.qg) + t * p.qg_st + (int64_t)h * 2 * hd
                      : static_cast<const T*>(p.k_new) + t * p.k_st + (int64_t)h * hd;
  float x[8];
  load_feat<T>(src + d0, x, dpl);
  float ss = 0.f;
  for (int e = 0; e < dpl; ++e) ss += x[e] * x[e];
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = 1.f / sqrtf(ss / (float)hd + p.eps);
  const float* wn = is_q ? p.q_norm : p.k_norm;
  float* xr = xs[warp];
  for (int e = 0; e < dpl; ++e) {
    x[e] = round_to<T>(x[e] * inv * wn[d0 + e]);
    xr[d0 + e] = x[e];
  }
  __syncwarp();
  const int half = p.rotary_dim / 2;
  T* dst = is_q ? static_cast<T*>(p.q_ws) + (t * p.heads + h) * hd + d0
                : static_cast<T*>(p.k_cache) + h * p.cache_sh + pos * hd + d0;
  for (int e = 0; e < dpl; ++e) {
    const int d = d0 + e;
    float y = x[e];
    if (d < p.rotary_dim) {
      const int i = d < half ? d : d - half;
      // angle = pos * base^(-2i / rotary_dim), reduced modulo 2 pi in double
      const double ang = remainder((double)pos * p.inv_freq[i], 6.283185307179586);
      float sn, cs;
      sincosf((float)ang, &sn, &cs);
      y = d < half ? x[e] * cs - xr[d + half] * sn : x[e] * cs + xr[d - half] * sn;
    }
    dst[e] = from_f<T>(y);
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
// four warps share each K/V tile (cp.async, double-buffered) and each owns
// kRows / kWarps rows with its own running max and sum.
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
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hk = blockIdx.y, split = blockIdx.z;
  const int64_t rows_all = p.n_tokens * p.group;
  const int64_t r0 = (int64_t)blockIdx.x * kRows;

  // the CTA's rows: (token, head) pairs of kv head hk, and their causal limits
  int64_t kmax = 0;
  for (int r = 0; r < kRows; ++r) {
    const int64_t R = r0 + r;
    if (R < rows_all) kmax = max(kmax, p.offset + R / p.group + 1);
  }
  int64_t lim[RPW];  // keys [0, lim) are visible to this warp's row i (0: inactive row)
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int64_t R = r0 + warp * RPW + i;
    lim[i] = R < rows_all ? p.offset + R / p.group + 1 : 0;
  }
  for (int i = tid; i < kRows * HD; i += kWarps * 32) {
    const int r = i / HD, d = i % HD;
    const int64_t R = r0 + r;
    float v = 0.f;
    if (R < rows_all) {
      const int64_t t = R / p.group;
      const int h = hk * p.group + (int)(R % p.group);
      v = to_f(static_cast<const T*>(p.q_ws)[(t * p.heads + h) * HD + d]);
    }
    qs[i] = v;
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
    for (int i = tid; i < nv * VPR; i += kWarps * 32) {
      const int row = i / VPR, col = (i % VPR) * SM::kVec;
      cp_async16((uint32_t)__cvta_generic_to_shared(kt + row * SM::kKRow + col), kc + (k0 + row) * HD + col, true);
      cp_async16((uint32_t)__cvta_generic_to_shared(vt + row * HD + col), vc + (k0 + row) * HD + col, true);
    }
  };
  if (ntiles > 0) issue(0);
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
    // scores: lane = key
    float s[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) s[i] = 0.f;
    if (lane < nvalid) {
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
            s[i] = fmaf(qv.x, kv[e], fmaf(qv.y, kv[e + 1], fmaf(qv.z, kv[e + 2], fmaf(qv.w, kv[e + 3], s[i]))));
          }
        }
      }
    }
    // online softmax per row
    const int64_t kpos = k0 + lane;
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const bool ok = lane < nvalid && kpos < lim[i];
      const float sv = ok ? s[i] * p.scale : -INFINITY;
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
    // output: lane = features [lane * DPL, +DPL)
    for (int j = 0; j < nvalid; ++j) {
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
    const int64_t R = r0 + warp * RPW + i;
    if (R >= rows_all) continue;
    const int64_t t = R / p.group;
    const int h = hk * p.group + (int)(R % p.group);
    const int64_t row = t * p.heads + h;
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
#pragma unroll
      for (int e = 0; e < DPL; ++e) pr[lane * DPL + e] = o[i][e];
      if (lane == 0) {
        pr[HD] = m[i];
        pr[HD + 1] = lsum[i];
      }
    }
  }
}

// Adds the splits' partial rows: out = sum_s e^(m_s - m) o_s / sum_s e^(m_s - m) l_s.
// One CTA per output row (token, head): warp 0 turns the splits' maxima and
// sums into weights in shared memory; the four warps then take every fourth
// split, each lane a run of head_dim / 32 features (16-byte loads, all of a
// warp's loads in flight), and their sums meet in shared memory.
constexpr int kMaxSplits = 160;

template <typename T>
__global__ void __launch_bounds__(128) attn_combine_kernel(const AttnParams p) {
  __shared__ float wsplit[kMaxSplits];
  __shared__ float inv_l;
  __shared__ __align__(16) float red[4][kMaxHeadDim];
  const int hd = p.head_dim, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t row = blockIdx.x;  // t * heads + h
  const size_t stride = (size_t)p.n_tokens * p.heads * (hd + 4);
  const float* base = p.part + row * (hd + 4);
  if (warp == 0) {
    float mm = -INFINITY;
    for (int s = lane; s < p.splits; s += 32) mm = fmaxf(mm, base[s * stride + hd]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, off));
    float l = 0.f;
    for (int s = lane; s < p.splits; s += 32) {
      const float ms = base[s * stride + hd];
      const float w = ms == -INFINITY ? 0.f : __expf(ms - mm);
      wsplit[s] = w;
      l += w * base[s * stride + hd + 1];
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (lane == 0) inv_l = 1.f / l;
  }
  __syncthreads();
  const int dpl = hd / 32;  // 1, 2, 4 or 8 features per lane
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int s = warp; s < p.splits; s += 4) {
    const float w = wsplit[s];
    const float* src = base + s * stride + lane * dpl;
    if (dpl >= 4) {
      const float4 a = reinterpret_cast<const float4*>(src)[0];
      acc[0] = fmaf(w, a.x, acc[0]);
      acc[1] = fmaf(w, a.y, acc[1]);
      acc[2] = fmaf(w, a.z, acc[2]);
      acc[3] = fmaf(w, a.w, acc[3]);
      if (dpl == 8) {
        const float4 b = reinterpret_cast<const float4*>(src)[1];
        acc[4] = fmaf(w, b.x, acc[4]);
        acc[5] = fmaf(w, b.y, acc[5]);
        acc[6] = fmaf(w, b.z, acc[6]);
        acc[7] = fmaf(w, b.w, acc[7]);
      }
    } else {
      for (int e = 0; e < dpl; ++e) acc[e] = fmaf(w, src[e], acc[e]);
    }
  }
  for (int e = 0; e < dpl; ++e) red[warp][lane * dpl + e] = acc[e];
  __syncthreads();
  const int64_t t = row / p.heads;
  const int h = (int)(row % p.heads);
  const T* gate = static_cast<const T*>(p.qg) + t * p.qg_st + (int64_t)h * 2 * hd + hd;
  T* dst = static_cast<T*>(p.out) + t * p.out_st + (int64_t)h * hd;
  for (int d = tid; d < hd; d += 128) {
    const float sum = red[0][d] + red[1][d] + red[2][d] + red[3][d];
    const float att = round_to<T>(sum * inv_l);
    const float gt = round_to<T>(sigmoid_f(to_f(gate[d])));
    dst[d] = from_f<T>(att * gt);
  }
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
  const int h = blockIdx.y, hk = h / p.group;
  const int64_t q0 = (int64_t)blockIdx.x * kMQ;  // first query (token index of this call)
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

template <int HD>
gdn_status launch_mma(const AttnParams& p, cudaStream_t s) {
  static bool attr = false;
  constexpr size_t smem = MmaSmem<HD>::kBytes;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_mma_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return set_error(GDN_ECUDA, "attention: shared-memory attribute");
    attr = true;
  }
  const dim3 grid((unsigned)((p.n_tokens + kMQ - 1) / kMQ), (unsigned)p.heads);
  attn_mma_kernel<HD><<<grid, kMmaThreads, smem, s>>>(p);
  return GDN_OK;
}

template <typename T, int HD>
gdn_status launch_fwd(const AttnParams& p, dim3 grid, cudaStream_t s) {
  static bool attr = false;  // set once per instance (a repeat from a racing thread is harmless)
  constexpr size_t smem = AttnSmem<T, HD>::kBytes;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_fwd_kernel<T, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return set_error(GDN_ECUDA, "attention: shared-memory attribute");
    attr = true;
  }
  attn_fwd_kernel<T, HD><<<grid, kWarps * 32, smem, s>>>(p);
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
    const int64_t max_by_keys = (a->cache_len + 2 * kKeyTile - 1) / (2 * kKeyTile);  // two tiles a split at least
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
  const size_t es = a->act_dtype == GDN_F32 ? 4 : 2;
  unsigned char* ws = static_cast<unsigned char*>(a->workspace);
  p.q_ws = ws;
  p.part = reinterpret_cast<float*>(ws + gdn::align256((size_t)a->n_tokens * a->heads * a->head_dim * es));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t prep_items = a->n_tokens * (a->heads + 2 * a->kv_heads);
  const dim3 pgrid((unsigned)((prep_items + gdn::kPrepWarps - 1) / gdn::kPrepWarps));
  const int64_t row_blocks = (a->n_tokens * p.group + gdn::kRows - 1) / gdn::kRows;
  if (row_blocks > 0x7fffffffLL) return gdn::set_error(GDN_EUNSUPPORTED, "too many rows for one call");
  const dim3 fgrid((unsigned)row_blocks, (unsigned)a->kv_heads, (unsigned)p.splits);
  if (a->act_dtype == GDN_F32) {
    gdn::attn_prep_kernel<float><<<pgrid, gdn::kPrepWarps * 32, 0, s>>>(p);
    st = gdn::launch_fwd_hd<float>(p, fgrid, s);
    if (st == GDN_OK && p.splits > 1) {
      gdn::attn_combine_kernel<float><<<(unsigned)(a->n_tokens * a->heads), 128, 0, s>>>(p);
    }
  } else {
    gdn::attn_prep_kernel<__nv_bfloat16><<<pgrid, gdn::kPrepWarps * 32, 0, s>>>(p);
    if (p.splits == 1 && a->head_dim >= 64) {  // prefill: the tensor-core kernel
      switch (a->head_dim) {
        case 64: st = gdn::launch_mma<64>(p, s); break;
        case 128: st = gdn::launch_mma<128>(p, s); break;
        default: st = gdn::launch_mma<256>(p, s); break;
      }
    } else {
      st = gdn::launch_fwd_hd<__nv_bfloat16>(p, fgrid, s);
    }
    if (st == GDN_OK && p.splits > 1) {
      gdn::attn_combine_kernel<__nv_bfloat16><<<(unsigned)(a->n_tokens * a->heads), 128, 0, s>>>(p);
    }
  }
  if (st != GDN_OK) return st;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return gdn::set_error(GDN_ECUDA, "attention launch: %s", cudaGetErrorString(e));
  return GDN_OK;
}
