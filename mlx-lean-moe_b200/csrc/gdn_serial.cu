// Token-serial gated-delta kernels: the single-token decode step and the
// general serial scan.  Both keep a tile of state rows in registers.
//
// Semantics (reference qw/gated_delta.py:24-41, per value head h, per token):
//     S <- g S;  r = S k;  d = beta (v - r);  S <- S + d k^T;  y = S q
// with S the (Dv, Dk) float32 state, Dk contiguous, and value head h reading
// key head h / (Hv / Hk) (qw/gated_delta.py:97-101).  (qw/ =
// src/mlx_lean_moe/model/qwen3_5/ in the reference project.)
//
// Register layout.  A state row (Dk floats) is split over LPR lanes of a
// warp, VEC float4 per lane, so one warp covers 32 / LPR rows at a time and
// a row's dot products reduce with log2(LPR) xor-shuffles inside its lane
// group.  Each load instruction of a warp covers 32/LPR rows x 16*LPR bytes,
// every sector used.  Each thread holds ITER row groups (ITER * VEC <= 8
// float4 of state) and issues all of their loads before any arithmetic, which
// is what keeps enough bytes in flight for HBM in the decode step.
#include <algorithm>

#include "gdn_common.cuh"

namespace gdn {
namespace {

// ITER_FIX > 0 sets the row groups per warp (decode at Dk = 128 takes four:
// sixteen 16-byte state loads in flight per thread).
template <int DKP, int ITER_FIX = 0>
struct Layout {
  static constexpr int LPR = DKP >= 32 ? 8 : DKP / 4;  // lanes per state row
  static constexpr int VEC = DKP / (4 * LPR);          // float4 per lane per row
  static constexpr int RPG = 32 / LPR;                 // rows per warp per group
  static constexpr int ITER_REG = VEC >= 8 ? 1 : 8 / VEC;
  static constexpr int ITER_CAP = 128 / (4 * RPG) > 0 ? 128 / (4 * RPG) : 1;
  static constexpr int ITER = ITER_FIX > 0 ? ITER_FIX : (ITER_REG < ITER_CAP ? ITER_REG : ITER_CAP);  // row groups per warp
  static constexpr int WARPS = 4;
  static constexpr int ROWS = WARPS * RPG * ITER;  // state rows per CTA
  static_assert(LPR * VEC * 4 == DKP, "layout");
};

template <int LPR>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int off = LPR / 2; off >= 1; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

__device__ __forceinline__ float load_gate(const void* base, gdn_dtype dt, int64_t idx) {
  return dt == GDN_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(base)[idx])
                        : static_cast<const float*>(base)[idx];
}

__device__ __forceinline__ void store_out(void* base, gdn_dtype dt, int64_t idx, float y) {
  if (dt == GDN_BF16)
    static_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(y);
  else
    static_cast<float*>(base)[idx] = y;
}

template <int DKP, typename T>
__device__ __forceinline__ float4 load_vec4(const T* row, int col, int dk) {
  if (col >= dk) return make_float4(0.f, 0.f, 0.f, 0.f);
  return make_float4(to_f(row[col]), to_f(row[col + 1]), to_f(row[col + 2]), to_f(row[col + 3]));
}

// One token for each of B sequences.  Grid: x = B * row tiles, y = Hv.
// Launched as a programmatic dependent of the kernel before it (typically the
// previous decode step): its CTAs become resident while that kernel drains
// and wait here before touching memory.  At Dk = 128, registers are capped
// for four CTAs per SM (128 a thread; 130 uncapped gave three): fewer,
// fuller waves of the 64-row tiles.
template <int DKP, typename T>
__global__ void __launch_bounds__(128, DKP == 128 ? 4 : 1) decode_kernel(const ScanParams p) {
  griddep_wait();  // launched as a dependent of the kernel before it
  griddep_launch_dependents();
  using L = Layout<DKP, DKP == 128 ? 4 : 0>;
  const int n_tiles = (p.dv + L::ROWS - 1) / L::ROWS;
  const int64_t b = blockIdx.x / n_tiles;
  const int tile = blockIdx.x % n_tiles;
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane / L::LPR, l = lane % L::LPR;
  const int kh = h / (p.hv / p.hk);
  const int dk = p.dk, dv = p.dv;

  const int64_t slot = p.state_slots ? (int64_t)p.state_slots[b] : b;
  const int64_t head_off = (slot * p.hv + h) * (int64_t)dv * dk;
  const int row0 = tile * L::ROWS + warp * (L::RPG * L::ITER) + grp;

  // Issue the state loads first: they are the bytes that matter.
  float4 s[L::ITER][L::VEC];
#pragma unroll
  for (int i = 0; i < L::ITER; ++i) {
    const int row = row0 + i * L::RPG;
#pragma unroll
    for (int j = 0; j < L::VEC; ++j) {
      const int col = (j * L::LPR + l) * 4;
      if (p.state_in && row < dv && col < dk)
        s[i][j] = *reinterpret_cast<const float4*>(p.state_in + head_off + (int64_t)row * dk + col);
      else
        s[i][j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }

  const T* kp = static_cast<const T*>(p.k) + b * p.k_st + kh * p.k_sh;
  const T* qp = static_cast<const T*>(p.q) + b * p.q_st + kh * p.q_sh;
  const T* vp = static_cast<const T*>(p.v) + b * p.v_st + h * p.v_sh;
  float4 kq[L::VEC], qq[L::VEC];
#pragma unroll
  for (int j = 0; j < L::VEC; ++j) {
    const int col = (j * L::LPR + l) * 4;
    kq[j] = load_vec4<DKP>(kp, col, dk);
    qq[j] = load_vec4<DKP>(qp, col, dk);
  }
  float gv = load_gate(p.g, p.gate_dtype, b * p.g_st + h);
  if (p.gate_kind == GDN_GATE_LOG) gv = expf(gv);
  const float bv = load_gate(p.beta, p.gate_dtype, b * p.beta_st + h);

  float* sout = p.state_out + head_off;
#pragma unroll
  for (int i = 0; i < L::ITER; ++i) {
    const int row = row0 + i * L::RPG;
    float r = 0.f;
#pragma unroll
    for (int j = 0; j < L::VEC; ++j) {
      s[i][j] = s[i][j] * gv;
      r += dot4(s[i][j], kq[j]);
    }
    r = group_sum<L::LPR>(r);
    const float vv = row < dv ? to_f(vp[row]) : 0.f;
    const float d = (vv - r) * bv;
    float y = 0.f;
#pragma unroll
    for (int j = 0; j < L::VEC; ++j) {
      s[i][j].x += kq[j].x * d;
      s[i][j].y += kq[j].y * d;
      s[i][j].z += kq[j].z * d;
      s[i][j].w += kq[j].w * d;
      y += dot4(s[i][j], qq[j]);
    }
    y = group_sum<L::LPR>(y);
    if (row < dv) {
#pragma unroll
      for (int j = 0; j < L::VEC; ++j) {
        const int col = (j * L::LPR + l) * 4;
        if (col < dk) *reinterpret_cast<float4*>(sout + (int64_t)row * dk + col) = s[i][j];
      }
      if (l == 0) store_out(p.out, p.out_dtype, (b * p.hv + h) * (int64_t)dv + row, y);
    }
  }
}

// Token-serial scan over packed sequences.  Grid: x = B * row tiles, y = Hv.
// q/k/v/g/beta of TB tokens are staged in shared memory (as float), then each
// thread advances its rows through those tokens with the state in registers.
// The next block of TB tokens is loaded into registers while the current one
// is processed, so global-memory latency stays off the token loop.
template <int DKP, typename T>
__global__ void __launch_bounds__(128) serial_scan_kernel(const ScanParams p) {
  griddep_wait();  // launched as a dependent of the kernel before it
  griddep_launch_dependents();
  using L = Layout<DKP>;
  constexpr int TB = DKP >= 256 ? 16 : 32;
  constexpr int NK = TB * DKP / 128;                       // k (and q) values staged per thread
  constexpr int NV = (TB * L::ROWS + 127) / 128;           // v values staged per thread
  static_assert(TB * DKP % 128 == 0, "staging layout");
  __shared__ __align__(16) float sk[TB][DKP];
  __shared__ __align__(16) float sq[TB][DKP];
  __shared__ float sv[TB][L::ROWS];
  __shared__ float sg[TB], sb[TB];

  const int n_tiles = (p.dv + L::ROWS - 1) / L::ROWS;
  const int64_t b = blockIdx.x / n_tiles;
  const int tile = blockIdx.x % n_tiles;
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane / L::LPR, l = lane % L::LPR;
  const int kh = h / (p.hv / p.hk);
  const int dk = p.dk, dv = p.dv;
  const int tile_row0 = tile * L::ROWS;
  const int local0 = warp * (L::RPG * L::ITER) + grp;  // this thread's first row within the tile

  int64_t start, end;
  seq_range(p.cu_seqlens, p.n_tokens, p.n_seqs, b, start, end);
  const int64_t head_off = (b * p.hv + h) * (int64_t)dv * dk;

  float4 s[L::ITER][L::VEC];
#pragma unroll
  for (int i = 0; i < L::ITER; ++i) {
    const int row = tile_row0 + local0 + i * L::RPG;
#pragma unroll
    for (int j = 0; j < L::VEC; ++j) {
      const int col = (j * L::LPR + l) * 4;
      if (p.state_in && row < dv && col < dk)
        s[i][j] = *reinterpret_cast<const float4*>(p.state_in + head_off + (int64_t)row * dk + col);
      else
        s[i][j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }

  const T* kbase = static_cast<const T*>(p.k) + kh * p.k_sh;
  const T* qbase = static_cast<const T*>(p.q) + kh * p.q_sh;
  const T* vbase = static_cast<const T*>(p.v) + h * p.v_sh;

  // Registers holding the next block of tokens.
  float pk[NK], pq[NK], pv[NV], pg = 0.f, pb = 0.f;
  auto prefetch = [&](int64_t t0) {
    const int64_t nt = end - t0 < TB ? end - t0 : TB;
#pragma unroll
    for (int e = 0; e < NK; ++e) {
      const int idx = threadIdx.x + 128 * e;
      const int tt = idx / DKP, c = idx % DKP;
      const bool ok = tt < nt && c < dk;
      pk[e] = ok ? to_f(kbase[(t0 + tt) * p.k_st + c]) : 0.f;
      pq[e] = ok ? to_f(qbase[(t0 + tt) * p.q_st + c]) : 0.f;
    }
#pragma unroll
    for (int e = 0; e < NV; ++e) {
      const int idx = threadIdx.x + 128 * e;
      const int tt = idx / L::ROWS, r = idx % L::ROWS;
      const int row = tile_row0 + r;
      pv[e] = (tt < nt && row < dv) ? to_f(vbase[(t0 + tt) * p.v_st + row]) : 0.f;
    }
    if (threadIdx.x < nt) {
      pg = load_gate(p.g, p.gate_dtype, (t0 + threadIdx.x) * p.g_st + h);
      if (p.gate_kind == GDN_GATE_LOG) pg = expf(pg);
      pb = load_gate(p.beta, p.gate_dtype, (t0 + threadIdx.x) * p.beta_st + h);
    }
  };

  if (start < end) prefetch(start);
  for (int64_t t0 = start; t0 < end; t0 += TB) {
    const int nt = (int)((end - t0) < TB ? (end - t0) : TB);
    __syncthreads();  // the previous block of tokens has been consumed
#pragma unroll
    for (int e = 0; e < NK; ++e) {
      const int idx = threadIdx.x + 128 * e;
      sk[idx / DKP][idx % DKP] = pk[e];
      sq[idx / DKP][idx % DKP] = pq[e];
    }
#pragma unroll
    for (int e = 0; e < NV; ++e) {
      const int idx = threadIdx.x + 128 * e;
      if (idx < TB * L::ROWS) sv[idx / L::ROWS][idx % L::ROWS] = pv[e];
    }
    if (threadIdx.x < TB) {
      sg[threadIdx.x] = pg;
      sb[threadIdx.x] = pb;
    }
    __syncthreads();
    if (t0 + TB < end) prefetch(t0 + TB);

    for (int tt = 0; tt < nt; ++tt) {
      const float gv = sg[tt], bv = sb[tt];
      float4 kq[L::VEC], qq[L::VEC];
#pragma unroll
      for (int j = 0; j < L::VEC; ++j) {
        kq[j] = reinterpret_cast<const float4*>(sk[tt])[j * L::LPR + l];
        qq[j] = reinterpret_cast<const float4*>(sq[tt])[j * L::LPR + l];
      }
#pragma unroll
      for (int i = 0; i < L::ITER; ++i) {
        const int local = local0 + i * L::RPG;
        const int row = tile_row0 + local;
        float r = 0.f;
#pragma unroll
        for (int j = 0; j < L::VEC; ++j) {
          s[i][j] = s[i][j] * gv;
          r += dot4(s[i][j], kq[j]);
        }
        r = group_sum<L::LPR>(r);
        const float d = (sv[tt][local] - r) * bv;
        float y = 0.f;
#pragma unroll
        for (int j = 0; j < L::VEC; ++j) {
          s[i][j].x += kq[j].x * d;
          s[i][j].y += kq[j].y * d;
          s[i][j].z += kq[j].z * d;
          s[i][j].w += kq[j].w * d;
          y += dot4(s[i][j], qq[j]);
        }
        y = group_sum<L::LPR>(y);
        if (row < dv && l == 0) store_out(p.out, p.out_dtype, ((t0 + tt) * p.hv + h) * (int64_t)dv + row, y);
      }
    }
  }

  float* sout = p.state_out + head_off;
#pragma unroll
  for (int i = 0; i < L::ITER; ++i) {
    const int row = tile_row0 + local0 + i * L::RPG;
    if (row >= dv) continue;
#pragma unroll
    for (int j = 0; j < L::VEC; ++j) {
      const int col = (j * L::LPR + l) * 4;
      if (col < dk) *reinterpret_cast<float4*>(sout + (int64_t)row * dk + col) = s[i][j];
    }
  }
}

int padded_dk(int dk) {
  int p = 4;
  while (p < dk) p <<= 1;
  return p;
}

template <int DKP, typename T>
cudaError_t launch_one(const ScanParams& p, cudaStream_t s, bool decode) {
  const int rows = decode ? Layout<DKP, DKP == 128 ? 4 : 0>::ROWS : Layout<DKP>::ROWS;
  const int64_t n_tiles = (p.dv + rows - 1) / rows;
  const int64_t gx = n_tiles * p.n_seqs;
  if (gx <= 0) return cudaSuccess;
  if (gx > 0x7fffffffLL || p.hv > 65535) return cudaErrorInvalidConfiguration;
  dim3 grid((unsigned)gx, (unsigned)p.hv);
  if (!decode) return launch_dependent(serial_scan_kernel<DKP, T>, grid, dim3(128), 0, s, p);
  return launch_dependent(decode_kernel<DKP, T>, grid, dim3(128), 0, s, p);
}

template <typename T>
cudaError_t dispatch_dk(const ScanParams& p, cudaStream_t s, bool decode) {
  switch (padded_dk(p.dk)) {
    case 4: return launch_one<4, T>(p, s, decode);
    case 8: return launch_one<8, T>(p, s, decode);
    case 16: return launch_one<16, T>(p, s, decode);
    case 32: return launch_one<32, T>(p, s, decode);
    case 64: return launch_one<64, T>(p, s, decode);
    case 128: return launch_one<128, T>(p, s, decode);
    case 256: return launch_one<256, T>(p, s, decode);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t dispatch(const ScanParams& p, cudaStream_t s, bool decode) {
  switch (p.qkv_dtype) {
    case GDN_F32: return dispatch_dk<float>(p, s, decode);
    case GDN_BF16: return dispatch_dk<__nv_bfloat16>(p, s, decode);
    case GDN_F16: return dispatch_dk<__half>(p, s, decode);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

bool serial_supported(int dk) { return dk >= 4 && dk <= 256 && dk % 4 == 0; }

cudaError_t launch_decode(const ScanParams& p, cudaStream_t s) { return dispatch(p, s, true); }
cudaError_t launch_serial_scan(const ScanParams& p, cudaStream_t s) { return dispatch(p, s, false); }

}  // namespace gdn
