// Chunked gated-delta prefill on the sm_100a tensor cores (chunk C = 64,
// Dk = Dv = 128, bf16 q/k/v, float32 state).
//
// The recurrence of the reference (qw/gated_delta.py:24-41, qw/ =
// src/mlx_lean_moe/model/qwen3_5/) run token by token is, over a chunk of C
// tokens with inclusive log-decay cumsum G (gamma = exp(G_last)):
//   A[t,s] = beta_t exp(G_t - G_s) k_t.k_s  (s < t),   T = (I + A)^-1
//   R      = diag(beta) (V - diag(exp G) K S^T)          (C x Dv)
//   Delta  = T R                                         (the d_t of every token)
//   Y      = diag(exp G) Q S^T + P Delta,  P[t,s] = exp(G_t - G_s) q_t.k_s (s <= t)
//   S'     = gamma S + Delta^T diag(exp(G_last - G)) K
// Every decay factor is exp of a difference G_t - G_s with t >= s (never a
// ratio of exponentials), so strong decays cannot overflow.
//
// Two kernels:
//  * chunk_prep_kernel, parallel over (chunk, value head): one tcgen05 MMA
//    [K;Q] K^T (M=128, N=64, K=128, bf16 inputs exact) gives K K^T and Q K^T
//    in TMEM; the epilogue builds A and P, a forward substitution gives T, and
//    T and P are written to the workspace as tf32 tiles in the SW128 K-major
//    operand layout.  The same kernel stores the chunk's gate vectors (beta,
//    exp G, exp(G_last - G), gamma) next to T and P.
//  * chunk_scan_kernel, one CTA per (sequence, value head), serial over the
//    chunks with the float32 state S resident in TMEM, read there as the tf32
//    A operand of the products that need it (no conversion of S on the
//    chain); see the kernel's own comment for the products and operands.
//  Precision: tf32 operands (S read with its low mantissa bits dropped, the
//  other tf32 operands rounded to nearest) and a bf16 hi + lo Delta' in the
//  state update give rel-L2 ~3e-4 to 5e-4 against the float64 recurrence at
//  T = 2048 in an emulation of these roundings, for slow, moderate and
//  strong decay.
//
// Every wait is bounded (2 s): on a timeout the kernel records an error in
// g_device_error (read by gdn_check_device_errors), stops issuing work, lets
// its own copies and MMAs in flight finish (again bounded), frees its TMEM
// and returns.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "gdn_common.cuh"
#include "gdn_sm100.cuh"

namespace gdn {

// Error word written by bounded device-side waits (0 = no error).
__device__ unsigned g_device_error = 0;

// Limit of every bounded wait in the chunked kernels (2 s unless a test
// shortens it through gdn_test_set_wait_limit), and the fault a test may
// inject (gdn_test_inject_fault; 0 = none).  Both are read once per CTA.
constexpr unsigned long long kDefaultWaitNs = 2000000000ull;
__device__ unsigned long long g_wait_limit_ns = kDefaultWaitNs;
__device__ int g_test_fault = 0;
constexpr int kFaultWithholdV = 1;  // the scan's producer never issues (nor arrives for) chunk 0's V tile

namespace {

using namespace sm100;

constexpr int CH = 64;   // chunk length
constexpr int DH = 128;  // head dim (Dk = Dv)
constexpr uint32_t kTileTf32 = 64 * 64 * 4;        // 64 x 64 tf32 operand tile (16 KB)
constexpr uint32_t kGateBytes = 1024;               // beta[64], exp G[64], exp(G_last - G)[64], gamma
// Per (chunk, head): T, P (tf32 [t][s], SW128 K-major), gates.
constexpr uint32_t kRecT = 0, kRecP = kTileTf32, kRecGates = 2 * kTileTf32;
constexpr size_t kRecBytes = 2 * (size_t)kTileTf32 + kGateBytes;
constexpr uint32_t GATE_BETA = 0, GATE_EG = 64, GATE_DG = 128, GATE_GAMMA = 192;  // float offsets

// A chain of the serial kernel other than "sequence b from state_in[b]":
// used to split one long sequence into segments (see launch_chunked_scan).
constexpr int kChainIdentity = 1;  // no state_in: start from the identity (a transition chain)
constexpr int kChainZeroV = 2;     // V taken as 0 (no V loads)
constexpr int kChainNoOut = 4;     // write no output
constexpr int kMaxChains = 16;
struct ChainDesc {
  int64_t seq;              // sequence (segment) of cu this chain runs over
  const float* state_in;    // [Hv, Dv, Dk] start state, or nullptr (0, or I with kChainIdentity)
  float* state_out;         // [Hv, Dv, Dk] final state, or nullptr (not written)
  int flags;
};

struct ChunkParams {
  int64_t n_tokens, n_seqs;
  const int64_t* cu;
  int hk, hv;
  const void* g;
  const void* beta;
  int64_t g_st, beta_st;
  gdn_dtype gate_dtype;
  gdn_gate_kind gate_kind;
  const float* state_in;
  float* state_out;
  void* out;
  gdn_dtype out_dtype;
  unsigned char* ws;  // kRecBytes per (chunk slot, value head)
  int64_t rec0;       // chunk prep: record index of its first slot (segments prepared apart)
  // Fused block: the output stage applies out = silu(z) * rms_norm(y -> bf16,
  // norm_w, eps) (z tiles by TMA), writing the layer output instead of y.
  int gated;
  const float* norm_w;
  float norm_eps;
  const __nv_bfloat16* z;  // [N, Hv, Dv] bf16, token stride z_st, head stride Dv
  int64_t z_st;
  // The output is [N, out_hv, Dv] with this call's heads at [head0, head0 +
  // hv); each output tile also goes to the n_peers other ranks' outputs.
  int out_hv, head0, n_peers;
  void* peer_out[GDN_MAX_GATHER_PEERS];
  // n_chains > 0: CTA row blockIdx.x / hv runs chains[row] instead of sequence
  // blockIdx.x / hv with state_in / state_out.
  int n_chains;
  ChainDesc chains[kMaxChains];
};

__device__ __forceinline__ float load_gate_f(const void* base, gdn_dtype dt, int64_t idx) {
  return dt == GDN_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(base)[idx])
                        : static_cast<const float*>(base)[idx];
}

// Log-decay of token t, head h (clamped so that cumulative sums stay finite).
__device__ __forceinline__ float log_decay(const ChunkParams& p, int64_t t, int h) {
  float x = load_gate_f(p.g, p.gate_dtype, t * p.g_st + h);
  if (p.gate_kind == GDN_GATE_MULT) x = logf(x);
  return fmaxf(x, -1.0e4f);
}

__device__ __forceinline__ int64_t nchunks_of(int64_t len) { return (len + CH - 1) / CH; }

// Chunk slot -> (sequence, chunk index within it); false past the last chunk.
// Warp-cooperative (every lane returns the same answer): 32 sequences per step.
__device__ bool slot_to_chunk(const ChunkParams& p, int64_t slot, int lane, int64_t& b, int64_t& j) {
  int64_t base = 0;
  for (int64_t s0 = 0; s0 < p.n_seqs; s0 += 32) {
    const int64_t s = s0 + lane;
    int64_t nc = 0;
    if (s < p.n_seqs) {
      int64_t st, en;
      seq_range(p.cu, p.n_tokens, p.n_seqs, s, st, en);
      nc = nchunks_of(en - st);
    }
    int64_t incl = nc;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int64_t o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    const int64_t excl = incl - nc;
    const unsigned hit = __ballot_sync(0xffffffffu, nc > 0 && slot >= base + excl && slot < base + incl);
    if (hit) {
      const int l = __ffs(hit) - 1;
      b = s0 + l;
      j = slot - base - __shfl_sync(0xffffffffu, excl, l);
      return true;
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
  return false;
}

__device__ int64_t chunk_base_of(const ChunkParams& p, int64_t b) {
  int64_t base = 0;
  for (int64_t s = 0; s < b; ++s) {
    int64_t st, en;
    seq_range(p.cu, p.n_tokens, p.n_seqs, s, st, en);
    base += nchunks_of(en - st);
  }
  return base;
}

// 32 consecutive gate values from shared memory (16-byte aligned) as float4s.
__device__ __forceinline__ void load_gate32(const float* src, float (&dst)[32]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 v = reinterpret_cast<const float4*>(src)[i];
    dst[4 * i] = v.x;
    dst[4 * i + 1] = v.y;
    dst[4 * i + 2] = v.z;
    dst[4 * i + 3] = v.w;
  }
}

__device__ __forceinline__ void record_error(volatile int* abort_flag) {
  *abort_flag = 1;
  atomicOr(&g_device_error, kErrTimeout);
}

// Inclusive prefix sum of sl[0..63] (log2 units) into sG by one warp (2
// values per lane); also exp(G), exp(G_last - G) and gamma = exp(G_last).
__device__ __forceinline__ void chunk_cumsum(int lane, const float* sl, float* sG, float* seG, float* sdG,
                                             float* sgamma) {
  float a = sl[2 * lane], b = sl[2 * lane + 1];
  float s = a + b;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const float o = __shfl_up_sync(0xffffffffu, s, off);
    if (lane >= off) s += o;
  }
  const float g1 = s, g0 = s - b;
  const float last = __shfl_sync(0xffffffffu, s, 31);
  sG[2 * lane] = g0;
  sG[2 * lane + 1] = g1;
  seG[2 * lane] = exp2f(g0);
  seG[2 * lane + 1] = exp2f(g1);
  sdG[2 * lane] = exp2f(last - g0);
  sdG[2 * lane + 1] = exp2f(last - g1);
  if (lane == 0) *sgamma = exp2f(last);
}

// ===========================================================================
// Kernel A: per (chunk, value head) -- T = (I + A)^-1 and P, as tf32 tiles.
// ===========================================================================
constexpr int kPrepAStride = 68;  // floats per row of the A / T scratch (16-byte rows)
// A and T scratch; it takes the place of the [K;Q] tile once the MMA has read it.
constexpr size_t kPrepScratch = 2 * 64 * kPrepAStride * 4;
static_assert(kPrepScratch >= 32768, "the scratch must cover the [K;Q] tile");
constexpr size_t kPrepSmem = 1024 + kPrepScratch;
constexpr float kLog2e = 1.4426950408889634f;

// Level-1 step of the doubling inverse for the 32-blocks (b0, b0+1):
// T[b1][b0] = -T[b1][b1] (A[b1][b0] T[b0][b0]), 16 x 16 blocks.  Thread tid
// (0..127) owns row ii, columns j0..j0+3 of one of the two pairs.
__device__ __forceinline__ void prep_level1(float* sA, float* sT, int tid) {
  const int pr = tid >> 6, ii = (tid >> 2) & 15, j0 = (tid & 3) * 4;
  const int r0 = 32 * pr, r1 = r0 + 16;  // first rows of blocks b0 and b1
  float2 m01 = make_float2(0.f, 0.f), m23 = make_float2(0.f, 0.f);
  const float* arow = sA + (r1 + ii) * kPrepAStride + r0;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float2 a = make_float2(arow[k], arow[k]);
    const float4 t4 = *reinterpret_cast<const float4*>(sT + (r0 + k) * kPrepAStride + r0 + j0);
    m01 = ffma2(a, make_float2(t4.x, t4.y), m01);
    m23 = ffma2(a, make_float2(t4.z, t4.w), m23);
  }
  // M -> the A[b0][b0] block (read only by the level-0 substitution, done).
  *reinterpret_cast<float4*>(sA + (r0 + ii) * kPrepAStride + r0 + j0) = make_float4(m01.x, m01.y, m23.x, m23.y);
  __syncthreads();
  float2 t01 = make_float2(0.f, 0.f), t23 = make_float2(0.f, 0.f);
  const float* trow = sT + (r1 + ii) * kPrepAStride + r1;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float2 tv = make_float2(trow[k], trow[k]);
    const float4 m4 = *reinterpret_cast<const float4*>(sA + (r0 + k) * kPrepAStride + r0 + j0);
    t01 = ffma2(tv, make_float2(m4.x, m4.y), t01);
    t23 = ffma2(tv, make_float2(m4.z, m4.w), t23);
  }
  *reinterpret_cast<float4*>(sT + (r1 + ii) * kPrepAStride + r0 + j0) = make_float4(-t01.x, -t01.y, -t23.x, -t23.y);
}

__global__ void __launch_bounds__(128, 6) chunk_prep_kernel(const __grid_constant__ CUtensorMap qmap,
                                                            const __grid_constant__ CUtensorMap kmap,
                                                            const ChunkParams p) {
  const uint64_t wait_ns = g_wait_limit_ns;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sKQ = base;                                        // [K;Q] 128 rows x 128, SW128
  float* sA = reinterpret_cast<float*>(base);                       // 64 x kPrepAStride (after the MMA)
  float* sT = sA + 64 * kPrepAStride;                               // 64 x kPrepAStride
  __shared__ __align__(16) float sl[CH], sb[CH], sG[CH], seG[CH], sdG[CH];
  __shared__ float sgamma;
  __shared__ __align__(8) uint64_t bar_load, bar_mma;
  __shared__ uint32_t tmem_base;
  __shared__ int64_t s_t0;
  __shared__ int s_n, s_valid;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.y;
  const int kh = h / (p.hv / p.hk);
  const int64_t slot = blockIdx.x;

  // The chunk's [K;Q] tile is requested as soon as its first token is known,
  // so that the load overlaps the tensor-memory allocation and gate reads.
  if (warp == 0) {
    int64_t b = 0, j = 0;
    const bool valid = slot_to_chunk(p, slot, lane, b, j);
    if (lane == 0) {
      s_valid = valid ? 1 : 0;
      abort_flag = 0;
      if (valid) {
        int64_t st, en;
        seq_range(p.cu, p.n_tokens, p.n_seqs, b, st, en);
        const int64_t c0 = st + j * CH;
        s_t0 = c0;
        s_n = (int)(en - c0 < CH ? en - c0 : CH);
        mbar_init(&bar_load, 1);
        mbar_init(&bar_mma, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(&bar_load, 32768);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          tma_load_3d(sKQ + kb * 16384, &kmap, &bar_load, kb * 64, kh, (int)c0);
          tma_load_3d(sKQ + kb * 16384 + 8192, &qmap, &bar_load, kb * 64, kh, (int)c0);
        }
      }
    }
  }
  __syncthreads();
  if (!s_valid) return;
  const int64_t t0 = s_t0;
  const int n = s_n;

  if (warp == 0) tmem_alloc(&tmem_base, 64);
  if (tid < CH) {
    const bool ok = tid < n;
    // Decays in log2 units: every exp below is an exp2 of a difference.
    sl[tid] = ok ? log_decay(p, t0 + tid, h) * kLog2e : 0.f;
    sb[tid] = ok ? load_gate_f(p.beta, p.gate_dtype, (t0 + tid) * p.beta_st + h) : 0.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 1) {
    chunk_cumsum(lane, sl, sG, seG, sdG, &sgamma);
    __syncwarp();
    float* gates = reinterpret_cast<float*>(p.ws + ((size_t)(p.rec0 + slot) * p.hv + h) * kRecBytes + kRecGates);
    for (int i = lane; i < CH; i += 32) {
      gates[GATE_BETA + i] = sb[i];
      gates[GATE_EG + i] = seG[i];
      gates[GATE_DG + i] = sdG[i];
    }
    for (int i = GATE_GAMMA + lane; i < (int)(kGateBytes / 4); i += 32) gates[i] = i == GATE_GAMMA ? sgamma : 0.f;
  }

  bool mma_issued = false;
  if (tid == 0) {
    if (mbar_wait(&bar_load, 0, wait_ns)) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16_f32(128, 64);
#pragma unroll
      for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t a = smem_u32(sKQ + kb * 16384 + ks * 32);
          mma_bf16(tmem, sdesc_sw128(a), sdesc_sw128(a), idesc, kb + ks > 0);
        }
      mma_commit(&bar_mma);
      mma_issued = true;
    } else {
      record_error(&abort_flag);
    }
  }
  __syncthreads();
  const bool ok = !abort_flag && mbar_wait(&bar_mma, 0, wait_ns);
  if (!ok && tid == 0) record_error(&abort_flag);
  __syncthreads();
  if (abort_flag) {
    if (tid == 0 && mma_issued) mbar_wait(&bar_mma, 0, wait_ns);
    if (tid == 0) mbar_wait(&bar_load, 0, wait_ns);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 64);
    return;
  }
  tc_fence_after();

  // Row r of [KK^T ; QK^T]: warps 0-1 hold K K^T rows, warps 2-3 Q K^T rows.
  // The [K;Q] tile is dead from here on: A and T take its place.
  const int row = warp * 32 + lane;
  float v[64];
  {
    const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16);
    tmem_ld32(ta, *reinterpret_cast<float(*)[32]>(v));
    tmem_ld32(ta + 32, *reinterpret_cast<float(*)[32]>(v + 32));
    tmem_wait_ld();
  }
  // Decay groups of four columns past the warp's last row are all masked
  // and skipped (warp-uniform).  ex2.approx (relative error ~2^-22) is far
  // below the tf32 resolution of the records.
  const int s_lim = (warp & 1) * 32 + 32;
  if (row < CH) {
    const int t = row;
    const float gt = sG[t], bt = sb[t];
    float* arow = sA + t * kPrepAStride;
#pragma unroll
    for (int s4 = 0; s4 < CH; s4 += 4) {
      float4 a4 = make_float4(0.f, 0.f, 0.f, 0.f);
      if (s4 < s_lim) {
        const float4 g4 = *reinterpret_cast<const float4*>(sG + s4);
        const float2 b2 = make_float2(bt, bt);
        const float2 p01 = fmul2(fmul2(b2, make_float2(ex2_approx(gt - g4.x), ex2_approx(gt - g4.y))),
                                 make_float2(v[s4], v[s4 + 1]));
        const float2 p23 = fmul2(fmul2(b2, make_float2(ex2_approx(gt - g4.z), ex2_approx(gt - g4.w))),
                                 make_float2(v[s4 + 2], v[s4 + 3]));
        a4.x = (s4 < t && t < n) ? p01.x : 0.f;
        a4.y = (s4 + 1 < t && t < n) ? p01.y : 0.f;
        a4.z = (s4 + 2 < t && t < n) ? p23.x : 0.f;
        a4.w = (s4 + 3 < t && t < n) ? p23.y : 0.f;
      }
      *reinterpret_cast<float4*>(arow + s4) = a4;
    }
  } else {
    const int t = row - CH;
    const float gt = sG[t];
#pragma unroll
    for (int s4 = 0; s4 < CH; s4 += 4) {
      if (s4 < s_lim) {
        const float4 g4 = *reinterpret_cast<const float4*>(sG + s4);
        const float2 p01 = fmul2(make_float2(ex2_approx(gt - g4.x), ex2_approx(gt - g4.y)), make_float2(v[s4], v[s4 + 1]));
        const float2 p23 =
            fmul2(make_float2(ex2_approx(gt - g4.z), ex2_approx(gt - g4.w)), make_float2(v[s4 + 2], v[s4 + 3]));
        v[s4] = (s4 <= t && t < n) ? p01.x : 0.f;
        v[s4 + 1] = (s4 + 1 <= t && t < n) ? p01.y : 0.f;
        v[s4 + 2] = (s4 + 2 <= t && t < n) ? p23.x : 0.f;
        v[s4 + 3] = (s4 + 3 <= t && t < n) ? p23.y : 0.f;
      } else {
        v[s4] = v[s4 + 1] = v[s4 + 2] = v[s4 + 3] = 0.f;
      }
    }
    // Row t of P as tf32: 16 chunks of 4, K-block j >> 3 (s in [32 kb, 32 kb + 32)).
    unsigned char* rec = p.ws + ((size_t)(p.rec0 + slot) * p.hv + h) * kRecBytes + kRecP;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      *reinterpret_cast<float4*>(rec + sw128_chunk(64, t, j >> 3, j & 7)) =
          make_float4(tf32_rn(v[4 * j]), tf32_rn(v[4 * j + 1]), tf32_rn(v[4 * j + 2]), tf32_rn(v[4 * j + 3]));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 64);

  // T = (I + A)^-1 by doubling.  Level 0: warp w inverts the diagonal 16-block
  // w by forward substitution (lane c < 16 owns column c); it also clears the
  // blocks of T above the diagonal that the later products read.
  {
    const int off = warp * 16, c = lane & 15;
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float* arow = sA + (off + i) * kPrepAStride + off;
      // (even, odd) partial sums as one pair; a missing odd term multiplies
      // 0 (A is finite, so the sum is unchanged)
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int j4 = 0; j4 < i; j4 += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(arow + j4);
        acc = ffma2(make_float2(a4.x, a4.y), make_float2(x[j4], j4 + 1 < i ? x[j4 + 1] : 0.f), acc);
        if (j4 + 2 < i) acc = ffma2(make_float2(a4.z, a4.w), make_float2(x[j4 + 2], j4 + 3 < i ? x[j4 + 3] : 0.f), acc);
      }
      x[i] = i < c ? 0.f : (i == c ? 1.f : -(acc.x + acc.y));
    }
    if (lane < 16) {
#pragma unroll
      for (int i = 0; i < 16; ++i) sT[(off + i) * kPrepAStride + off + c] = x[i];
      if ((warp & 1) == 0) {
#pragma unroll
        for (int i = 0; i < 16; ++i) sT[(off + i) * kPrepAStride + off + 16 + c] = 0.f;
      }
    }
    if (warp < 2) {
#pragma unroll
      for (int i = 0; i < 16; ++i) sT[(off + i) * kPrepAStride + 32 + lane] = 0.f;  // T12
    }
  }
  __syncthreads();
  // Level 1: the two diagonal 32-blocks.
  prep_level1(sA, sT, tid);
  __syncthreads();
  // Level 2: T21 = -T22 (A21 T11) with M = A21 T11 in the (dead) A11 block.
  {
    const int i = tid >> 2, j0 = (tid & 3) * 8;
    float2 m[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    const float* arow = sA + (32 + i) * kPrepAStride;
#pragma unroll 2
    for (int k4 = 0; k4 < 32; k4 += 4) {
      const float4 a4 = *reinterpret_cast<const float4*>(arow + k4);
      const float a[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float4 t0v = *reinterpret_cast<const float4*>(sT + (k4 + kk) * kPrepAStride + j0);
        const float4 t1v = *reinterpret_cast<const float4*>(sT + (k4 + kk) * kPrepAStride + j0 + 4);
        const float2 aa = make_float2(a[kk], a[kk]);
        m[0] = ffma2(aa, make_float2(t0v.x, t0v.y), m[0]);
        m[1] = ffma2(aa, make_float2(t0v.z, t0v.w), m[1]);
        m[2] = ffma2(aa, make_float2(t1v.x, t1v.y), m[2]);
        m[3] = ffma2(aa, make_float2(t1v.z, t1v.w), m[3]);
      }
    }
    __syncthreads();
    *reinterpret_cast<float4*>(sA + i * kPrepAStride + j0) = make_float4(m[0].x, m[0].y, m[1].x, m[1].y);
    *reinterpret_cast<float4*>(sA + i * kPrepAStride + j0 + 4) = make_float4(m[2].x, m[2].y, m[3].x, m[3].y);
  }
  __syncthreads();
  {
    const int i = tid >> 2, j0 = (tid & 3) * 8;
    float2 m[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    const float* trow = sT + (32 + i) * kPrepAStride + 32;
#pragma unroll 2
    for (int k4 = 0; k4 < 32; k4 += 4) {
      const float4 t4 = *reinterpret_cast<const float4*>(trow + k4);
      const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float4 m0v = *reinterpret_cast<const float4*>(sA + (k4 + kk) * kPrepAStride + j0);
        const float4 m1v = *reinterpret_cast<const float4*>(sA + (k4 + kk) * kPrepAStride + j0 + 4);
        const float2 tt = make_float2(tv[kk], tv[kk]);
        m[0] = ffma2(tt, make_float2(m0v.x, m0v.y), m[0]);
        m[1] = ffma2(tt, make_float2(m0v.z, m0v.w), m[1]);
        m[2] = ffma2(tt, make_float2(m1v.x, m1v.y), m[2]);
        m[3] = ffma2(tt, make_float2(m1v.z, m1v.w), m[3]);
      }
    }
    *reinterpret_cast<float4*>(sT + (32 + i) * kPrepAStride + j0) = make_float4(-m[0].x, -m[0].y, -m[1].x, -m[1].y);
    *reinterpret_cast<float4*>(sT + (32 + i) * kPrepAStride + j0 + 4) =
        make_float4(-m[2].x, -m[2].y, -m[3].x, -m[3].y);
  }
  __syncthreads();
  {
    // Row t, K-block kb (s in [32 kb, 32 kb + 32)) of T as tf32.
    const int t = tid & 63, kb = tid >> 6;
    unsigned char* rec = p.ws + ((size_t)(p.rec0 + slot) * p.hv + h) * kRecBytes + kRecT;
    const float* trow = sT + t * kPrepAStride + 32 * kb;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 x = *reinterpret_cast<const float4*>(trow + 4 * c);
      *reinterpret_cast<float4*>(rec + sw128_chunk(64, t, kb, c)) =
          make_float4(tf32_rn(x.x), tf32_rn(x.y), tf32_rn(x.z), tf32_rn(x.w));
    }
  }
}

// ===========================================================================
// Kernel B: per (sequence, value head) -- serial over chunks, S in TMEM.
// ===========================================================================
// The float32 state S lives in TMEM and never leaves it during the scan: the
// X|Y product reads it there as its tf32 A operand (kind::tf32 with a TMEM A
// operand).  Per chunk, in the transposed orientation (M = 128 state rows
// dv), with b the chunk's parity:
//   [X | Y]_b = S [K ; Q~]^T     tf32, N = 128, K = Dk   Q~ = diag(e^G) Q, so y = Y + O
//   R   = diag(beta)(V - diag(e^G) X)                     over X, rounded to tf32
//   D_b = R^T T^T (= Delta^T)    tf32, N = 64, K = C
//   S   = gamma S + Delta'^T K   bf16, N = Dk, K = C: Delta' = Delta diag(e^(G_last - G)) as
//                                bf16 hi + lo over the dead R; K (exact in bf16) read
//                                MN-major from its TMA tile
//   Y_b += D_b P^T               tf32, N = 64, K = C     issued a chunk later, off the chain
// The chain per chunk is X|Y -> R -> Delta -> Delta' -> S.  [X|Y] and Delta
// are double-buffered by parity, so neither the output warps nor the late O
// product hold the chain up.  Four converter warps widen K and Q from their
// bf16 tiles into the one fp32 [K ; Q~] operand tile (Q scaled by e^G).
//
// Dynamic shared memory (offsets from the 1024-aligned base).  fp32 operand
// tiles are SW128 K-major: per K-block of 32 floats, one 128-byte row each.
constexpr uint32_t kBTile = 64 * DH * 2;             // bf16 [64 t][128] tile (16 KB)
constexpr uint32_t OFF_KQ = 0;                        // fp32 [K ; Q~] 128 rows x 128: 4 K-blocks of 16 KB
constexpr uint32_t OFF_KB = 4 * 128 * 128;            // bf16 K TMA tiles (SW128), chunk parity
constexpr uint32_t OFF_QB = OFF_KB + 2 * kBTile;      // bf16 Q TMA tile (SW128)
constexpr uint32_t OFF_V = OFF_QB + kBTile;           // V bf16 [64 t][128 dv] row-major
constexpr uint32_t OFF_T = OFF_V + kBTile;            // T [t][s] tf32 (16 KB)
constexpr uint32_t OFF_P = OFF_T + kTileTf32;         // P [t][s] tf32 (16 KB)
constexpr uint32_t OFF_GATES = OFF_P + kTileTf32;     // two 1 KB gate buffers (chunk parity)
constexpr uint32_t OFF_OSTAGE = OFF_GATES + 2 * kGateBytes;  // output staging [64 t][128 dv], out dtype
constexpr uint32_t OFF_Z = OFF_OSTAGE + 64 * DH * 4;          // gated output: z [64 t][128 dv] bf16 (TMA)
constexpr uint32_t SCAN_SMEM_USED = OFF_Z + kBTile;
constexpr size_t kScanSmem = 1024 + SCAN_SMEM_USED;
static_assert(OFF_KB % 1024 == 0 && OFF_QB % 1024 == 0 && OFF_T % 1024 == 0 && OFF_P % 1024 == 0,
              "operand tiles on 1 KB boundaries");
static_assert(OFF_OSTAGE % 128 == 0, "TMA store source on 128 B");
constexpr int kScanThreads = 576;
constexpr int kEpiThreads = 256;                   // warps 2-9: the state chain
constexpr int kOutThreads = 128;                   // warps 10-13: the output
constexpr int kCvtThreads = 128;                   // warps 14-17: bf16 -> tf32 operand tile

// TMEM columns (512): S, then [X | Y] of each parity (X's 64 columns hold R,
// then Delta' hi / lo), then Delta of each parity.
constexpr uint32_t TM_S = 0, TM_XY = 128, TM_D = 384;

enum Bar {
  B_K_FULL0, B_K_FULL1, B_K_EMPTY0, B_K_EMPTY1, B_KQ_READY,
  B_Q_FULL, B_Q_EMPTY, B_V_FULL, B_V_EMPTY, B_T_FULL, B_T_EMPTY, B_P_FULL, B_P_EMPTY,
  B_S_INIT, B_X_DONE, B_R_READY, B_D_DONE, B_DD_READY, B_DR_READY, B_U_DONE,
  B_OU_DONE0, B_OU_DONE1, B_Y_FREE0, B_Y_FREE1, B_Z_FULL,
  B_DRAIN,
  N_BARS
};

// Copies rows 0 .. n-1 of a staged output tile ([t][Dv] rows of the out
// dtype, contiguous) of value head h, tokens t0 .., to every peer's gathered
// output: 16-byte loads from shared memory, one 16-byte store per peer (over
// NVLink for another GPU's memory).  The 128 output threads, thread e.
__device__ __forceinline__ void copy_tile_to_peers(const ChunkParams& p, const unsigned char* stage, int64_t t0,
                                                   int n, int h, int e) {
  const int row_chunks = DH * (p.out_dtype == GDN_BF16 ? 2 : 4) / 16;
  const int total = n * row_chunks;
  for (int i = e; i < total; i += 128) {
    const int r = i / row_chunks, c = i - r * row_chunks;
    const uint4 v = reinterpret_cast<const uint4*>(stage)[i];
    const size_t off = (((size_t)(t0 + r) * p.out_hv + p.head0 + h) * row_chunks + c) * 16;
    for (int j = 0; j < p.n_peers; ++j) *reinterpret_cast<uint4*>(static_cast<unsigned char*>(p.peer_out[j]) + off) = v;
  }
}

// Widens a bf16 [64 t][128] SW128 tile (two 64-wide K-blocks, 16 KB at src)
// into rows row0 .. row0 + 63 of the 128-row fp32 SW128 K-major tile at dst,
// row t scaled by scale[t] and rounded to tf32 when scale is given.  128
// threads, thread e; each moves eight 16-byte chunks.
__device__ __forceinline__ void widen_tile(const unsigned char* src, unsigned char* dst, int row0, const float* scale,
                                           int e) {
  uint4 raw[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) raw[j] = reinterpret_cast<const uint4*>(src)[e + 128 * j];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int i = e + 128 * j;                  // physical 16-byte chunk of the bf16 tile
    const int kb = i >> 9, r = (i >> 3) & 63;   // 64-wide K-block, row
    const int c = (i & 7) ^ (r & 7);            // logical chunk: elements 64 kb + 8 c .. + 7
    const uint32_t w[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
    float f[8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      f[2 * u] = bf16_lo_f(w[u]);
      f[2 * u + 1] = bf16_hi_f(w[u]);
    }
    if (scale) {
      const float s = scale[r];
#pragma unroll
      for (int u = 0; u < 8; ++u) f[u] = tf32_rn(f[u] * s);
    }
    const int fb = 2 * kb + (c >> 2), cc = 2 * (c & 3);
    *reinterpret_cast<float4*>(dst + sw128_chunk(128, row0 + r, fb, cc)) = make_float4(f[0], f[1], f[2], f[3]);
    *reinterpret_cast<float4*>(dst + sw128_chunk(128, row0 + r, fb, cc + 1)) = make_float4(f[4], f[5], f[6], f[7]);
  }
}

// GATHER: the output goes into a [N, out_hv, Dv] gathered output at head0 and
// to the peers' (gdn_scan_gathered); a separate instance, so that the plain
// scan's code is not touched by it.
template <bool GATHER>
__global__ void __launch_bounds__(kScanThreads, 1) chunk_scan_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                     const __grid_constant__ CUtensorMap kmap,
                                                                     const __grid_constant__ CUtensorMap vmap,
                                                                     const __grid_constant__ CUtensorMap omap,
                                                                     const __grid_constant__ CUtensorMap zmap,
                                                                     const ChunkParams p) {
  const uint64_t wait_ns = g_wait_limit_ns;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bars[N_BARS];
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ int64_t s_start, s_end, s_cbase;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x % p.hv;
  const int64_t row = blockIdx.x / p.hv;
  const int kh = h / (p.hv / p.hk);
  const size_t head_state = (size_t)h * DH * DH;
  int64_t b;
  const float* chain_in;
  float* chain_out;
  int flags;
  if (p.n_chains > 0) {
    const ChainDesc& d = p.chains[row];
    b = d.seq;
    chain_in = d.state_in ? d.state_in + head_state : nullptr;
    chain_out = d.state_out ? d.state_out + head_state : nullptr;
    flags = d.flags;
  } else {
    b = row;
    const size_t off = (size_t)b * p.hv * DH * DH + head_state;
    chain_in = p.state_in ? p.state_in + off : nullptr;
    chain_out = p.state_out + off;
    flags = 0;
  }
  if (flags & kChainZeroV) {  // V = 0 for a transition chain: a zero tile, never loaded
    for (int i = tid; i < (int)(kBTile / 16); i += blockDim.x)
      reinterpret_cast<uint4*>(base + OFF_V)[i] = make_uint4(0u, 0u, 0u, 0u);
  }

  if (tid == 0) {
    int64_t st, en;
    seq_range(p.cu, p.n_tokens, p.n_seqs, b, st, en);
    s_start = st;
    s_end = en;
    s_cbase = chunk_base_of(p, b);
    abort_flag = 0;
    for (int i = 0; i < N_BARS; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const int64_t start = s_start, end = s_end;
  const int64_t nch = nchunks_of(end - start);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Lane 0 keeps five operand streams going -- K (bf16, two buffers) with
    // the gates, Q, V, T, P -- each in chunk order, each load issued as soon
    // as the chunk before is done with that buffer.  It polls the streams
    // round-robin with non-blocking tests, never waiting on any one of them (a
    // late consumer of one buffer must not hold up the loads of the others),
    // and gives up (recording a timeout) once no stream has advanced for the
    // wait limit.  With each K load it prefetches chunk c + 2's tiles and
    // records into L2, so the loads themselves arrive at L2 latency.
    if (nch > 0 && lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      prefetch_tensormap(&omap);
      if (p.gated) prefetch_tensormap(&zmap);
      const bool withhold_v = g_test_fault == kFaultWithholdV;
      int64_t next[5] = {0, 0, 0, 0, 0};   // next chunk to load, per stream
      uint32_t n_k[2] = {0, 0};            // K loads issued per buffer
      uint64_t last = globaltimer_ns();
      while (!abort_flag) {
        bool progress = false, pending = false;
        for (int sidx = 0; sidx < 5; ++sidx) {
          const int64_t c = next[sidx];
          if (c >= nch) continue;
          pending = true;
          const int bb = (int)(c & 1);
          const uint32_t par = (uint32_t)((c - 1) & 1);
          const int t0 = (int)(start + c * CH);
          const unsigned char* rec = p.ws + ((size_t)(s_cbase + c) * p.hv + h) * kRecBytes;
          if (sidx == 0) {  // K_c and the gates into buffer c & 1, free once U_(c-2) is done
            if (c >= 2 && !mbar_test_wait(&bars[B_K_EMPTY0 + bb], (uint32_t)(((c >> 1) - 1) & 1))) continue;
            if (c + 2 < nch) {
              const int t2 = t0 + 2 * CH;
              tma_prefetch_3d(&kmap, 0, kh, t2);
              tma_prefetch_3d(&kmap, 64, kh, t2);
              tma_prefetch_3d(&qmap, 0, kh, t2);
              tma_prefetch_3d(&qmap, 64, kh, t2);
              if (!(flags & kChainZeroV)) tma_prefetch_3d(&vmap, 0, h, t2);
              if (p.gated && !(flags & kChainNoOut)) tma_prefetch_3d(&zmap, 0, h, t2);
              bulk_prefetch_l2(rec + 2 * (size_t)p.hv * kRecBytes, (uint32_t)kRecBytes);
            }
            mbar_arrive_expect_tx(&bars[B_K_FULL0 + bb], kBTile + kGateBytes);
            tma_load_3d(base + OFF_KB + bb * kBTile, &kmap, &bars[B_K_FULL0 + bb], 0, kh, t0);
            tma_load_3d(base + OFF_KB + bb * kBTile + 8192, &kmap, &bars[B_K_FULL0 + bb], 64, kh, t0);
            bulk_load(base + OFF_GATES + bb * kGateBytes, rec + kRecGates, kGateBytes, &bars[B_K_FULL0 + bb]);
            ++n_k[bb];
          } else if (sidx == 1) {  // Q_c once the converter has read Q_(c-1)
            if (c >= 1 && !mbar_test_wait(&bars[B_Q_EMPTY], par)) continue;
            mbar_arrive_expect_tx(&bars[B_Q_FULL], kBTile);
            tma_load_3d(base + OFF_QB, &qmap, &bars[B_Q_FULL], 0, kh, t0);
            tma_load_3d(base + OFF_QB + 8192, &qmap, &bars[B_Q_FULL], 64, kh, t0);
          } else if (sidx == 2) {  // V_c once R_(c-1) has read V_(c-1)
            if (c >= 1 && !mbar_test_wait(&bars[B_V_EMPTY], par)) continue;
            if (withhold_v && c == 0) {
              // test fault: V_FULL never completes, so the waits on it run out
            } else if (flags & kChainZeroV) {
              mbar_arrive(&bars[B_V_FULL]);
            } else {
              mbar_arrive_expect_tx(&bars[B_V_FULL], kBTile);
              tma_load_3d(base + OFF_V, &vmap, &bars[B_V_FULL], 0, h, t0);
            }
          } else if (sidx == 3) {  // T_c once Delta_(c-1) has read T_(c-1)
            if (c >= 1 && !mbar_test_wait(&bars[B_T_EMPTY], par)) continue;
            mbar_arrive_expect_tx(&bars[B_T_FULL], kTileTf32);
            bulk_load(base + OFF_T, rec + kRecT, kTileTf32, &bars[B_T_FULL]);
          } else {  // P_c once O_(c-1) has read P_(c-1)
            if (c >= 1 && !mbar_test_wait(&bars[B_P_EMPTY], par)) continue;
            mbar_arrive_expect_tx(&bars[B_P_FULL], kTileTf32);
            bulk_load(base + OFF_P, rec + kRecP, kTileTf32, &bars[B_P_FULL]);
          }
          next[sidx] = c + 1;
          progress = true;
        }
        if (!pending) break;
        const uint64_t now = globaltimer_ns();
        if (progress) {
          last = now;
        } else if (now - last > wait_ns) {
          record_error(&abort_flag);
          break;
        }
      }
      // After an abort, let the copies this thread started land (bounded)
      // before the CTA releases its shared memory.  Stream s has issued
      // next[s] loads (V one fewer when the test fault withheld chunk 0's).
      if (abort_flag) {
        for (int bb = 0; bb < 2; ++bb)
          if (n_k[bb]) mbar_wait(&bars[B_K_FULL0 + bb], (n_k[bb] - 1) & 1, wait_ns);
        if (next[1]) mbar_wait(&bars[B_Q_FULL], (uint32_t)((next[1] - 1) & 1), wait_ns);
        const int64_t nv = next[2] - (withhold_v && next[2] > 0 ? 1 : 0);
        if (nv > 0) mbar_wait(&bars[B_V_FULL], (uint32_t)((nv - 1) & 1), wait_ns);
        if (next[3]) mbar_wait(&bars[B_T_FULL], (uint32_t)((next[3] - 1) & 1), wait_ns);
        if (next[4]) mbar_wait(&bars[B_P_FULL], (uint32_t)((next[4] - 1) & 1), wait_ns);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Per chunk: [X|Y]_c (the chain), O_(c-1), Delta_c, U_c.  A product that
    // reads a TMEM operand written by the epilogue or by an earlier product is
    // issued after the barrier that says that operand is complete.
    if (lane == 0 && nch > 0) {
      const uint32_t id128 = idesc_tf32_f32(128, 128);
      const uint32_t id64 = idesc_tf32_f32(128, 64);
      const uint32_t idu = idesc_bf16_f32_bmn(128, 128);
      const uint32_t sKQ = smem_u32(base + OFF_KQ);
      const uint32_t sKb[2] = {smem_u32(base + OFF_KB), smem_u32(base + OFF_KB + kBTile)};
      const uint32_t sT = smem_u32(base + OFF_T), sP = smem_u32(base + OFF_P);
      // O_c^T += Delta_c^T P_c^T onto Y of chunk c's parity, in two halves
      // of K (tokens 0-31, 32-63) placed where the tensor pipe would idle;
      // the first half waits for the rounded Delta_c and P_c.
      auto issue_o = [&](int64_t c, int part) -> bool {
        if (part == 0 && (!mbar_wait(&bars[B_P_FULL], (uint32_t)(c & 1), wait_ns) ||
                          !mbar_wait(&bars[B_DR_READY], (uint32_t)(c & 1), wait_ns)))
          return false;
        tc_fence_after();
        const uint32_t cb = (uint32_t)(c & 1);
        for (int ks = 4 * part; ks < 4 * part + 4; ++ks)
          mma_tf32_ts(tmem + TM_XY + 128 * cb + 64, tmem + TM_D + 64 * cb + 8 * ks,
                      sdesc_sw128(sP + (ks >> 2) * 8192 + (ks & 3) * 32), id64, true);
        if (part == 1) {
          mma_commit(&bars[B_OU_DONE0 + cb]);
          mma_commit(&bars[B_P_EMPTY]);
        }
        return true;
      };
      bool ok = mbar_wait(&bars[B_S_INIT], 0, wait_ns);
      for (int64_t c = 0; ok && c < nch; ++c) {
        const int bb = (int)(c & 1);
        const uint32_t par = (uint32_t)(c & 1);
        const uint32_t xy = tmem + TM_XY + 128 * (uint32_t)bb;
        // [X|Y]_c = S [K ; Q~]_c^T, S as left by U_(c-1), into the region the
        // output warps have finished with (chunk c - 2's Y)
        ok = mbar_wait(&bars[B_KQ_READY], par, wait_ns) &&
             (c == 0 || mbar_wait_spin(&bars[B_U_DONE], (uint32_t)((c - 1) & 1), wait_ns)) &&
             (c < 2 || mbar_wait(&bars[B_Y_FREE0 + bb], (uint32_t)(((c >> 1) - 1) & 1), wait_ns));
        if (!ok || abort_flag) break;
        tc_fence_after();
        for (int ks = 0; ks < 16; ++ks)
          mma_tf32_ts(xy, tmem + TM_S + 8 * ks, sdesc_sw128(sKQ + (ks >> 2) * 16384 + (ks & 3) * 32), id128, ks > 0);
        mma_commit(&bars[B_X_DONE]);
        // first half of O_(c-1) right behind it: it runs while the epilogue
        // forms R, when the tensor pipe would otherwise idle
        if (c > 0 && !(ok = issue_o(c - 1, 0))) break;
        // D_b = Delta_c^T = R^T T^T (R over X)
        ok = mbar_wait(&bars[B_T_FULL], par, wait_ns) && mbar_wait_spin(&bars[B_R_READY], par, wait_ns);
        if (!ok || abort_flag) break;
        tc_fence_after();
        for (int ks = 0; ks < 8; ++ks)
          mma_tf32_ts(tmem + TM_D + 64 * bb, xy + 8 * ks, sdesc_sw128(sT + (ks >> 2) * 8192 + (ks & 3) * 32), id64,
                      ks > 0);
        mma_commit(&bars[B_D_DONE]);
        mma_commit(&bars[B_T_EMPTY]);
        // second half of O_(c-1), while the epilogue forms Delta'
        if (c > 0 && !(ok = issue_o(c - 1, 1))) break;
        // S = gamma S + Delta'^T K: Delta' hi then lo (packed bf16 over X),
        // K from its bf16 TMA tile read MN-major (N = Dk contiguous)
        ok = mbar_wait_spin(&bars[B_DD_READY], par, wait_ns);
        if (!ok || abort_flag) break;
        tc_fence_after();
        for (int part = 0; part < 2; ++part)
          for (int ks = 0; ks < 4; ++ks)
            mma_bf16_ts(tmem + TM_S, xy + 32 * part + 8 * ks, sdesc_sw128_mn(sKb[bb] + ks * 2048, 8192, 1024), idu,
                        true);
        mma_commit(&bars[B_U_DONE]);
        mma_commit(&bars[B_K_EMPTY0 + bb]);
      }
      if (ok && !abort_flag) ok = issue_o(nch - 1, 0) && issue_o(nch - 1, 1);
      if (!ok) record_error(&abort_flag);
      // Wait for every MMA issued so far before the CTA winds down.
      mma_commit(&bars[B_DRAIN]);
      mbar_wait(&bars[B_DRAIN], 0, wait_ns);
    }
  } else if (warp < 10) {
    // ------------------------------------------------------- state-chain epilogue
    const int e = tid - 64;                   // 0..255
    const int q = warp & 3;                   // TMEM lane quarter of this warp
    const int half = (warp - 2) >> 2;         // which half of the columns this thread owns
    const int dv = q * 32 + lane;             // state row
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    const bool leader = e == 0;
    unsigned char* sm = base;

    // S_0 -> TMEM: columns 64 half .. + 63 of row dv.
    {
      const float* srow = chain_in ? chain_in + (size_t)dv * DH : nullptr;
      const float diag = (flags & kChainIdentity) ? 1.f : 0.f;
      for (int cc = 0; cc < 2; ++cc) {
        const int col = half * 64 + cc * 32;
        float x[32];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 v4 = srow ? *reinterpret_cast<const float4*>(srow + col + i) : make_float4(0.f, 0.f, 0.f, 0.f);
          x[i] = v4.x;
          x[i + 1] = v4.y;
          x[i + 2] = v4.z;
          x[i + 3] = v4.w;
        }
        if (!srow) {
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = (col + i == dv) ? diag : 0.f;
        }
        tmem_st32(tq + TM_S + col, x);
      }
      tmem_wait_st();
      tc_fence_before();
      named_sync(1, kEpiThreads);
      if (leader) mbar_arrive(&bars[B_S_INIT]);
    }

    for (int64_t c = 0; c < nch; ++c) {
      const uint32_t par = (uint32_t)(c & 1);
      const uint32_t cb = (uint32_t)(c & 1);
      const uint32_t xq = tq + TM_XY + 128 * cb;  // this chunk's [X|Y] region, this warp's lanes
      const float* gates = reinterpret_cast<const float*>(sm + OFF_GATES + cb * kGateBytes);

      // beta V of tokens 32 half .. + 31 ahead of X, then
      // R = beta V - (beta e^G) X over X.
      bool ok = mbar_wait(&bars[B_K_FULL0 + cb], (uint32_t)((c >> 1) & 1), wait_ns) &&  // the gates
                mbar_wait(&bars[B_V_FULL], par, wait_ns);
      if (!ok) record_error(&abort_flag);
      if (named_sync_or(1, kEpiThreads, !ok)) break;
      float bv[32];
      {
        const __nv_bfloat16* V = reinterpret_cast<const __nv_bfloat16*>(sm + OFF_V) + dv;
#pragma unroll
        for (int i4 = 0; i4 < 32; i4 += 4) {
          const float4 b4 = *reinterpret_cast<const float4*>(gates + GATE_BETA + half * 32 + i4);
          const int t = half * 32 + i4;
          bv[i4] = b4.x * __bfloat162float(V[t * DH]);
          bv[i4 + 1] = b4.y * __bfloat162float(V[(t + 1) * DH]);
          bv[i4 + 2] = b4.z * __bfloat162float(V[(t + 2) * DH]);
          bv[i4 + 3] = b4.w * __bfloat162float(V[(t + 3) * DH]);
        }
      }
      ok = mbar_wait(&bars[B_X_DONE], par, wait_ns);
      if (!ok) record_error(&abort_flag);
      if (named_sync_or(1, kEpiThreads, !ok)) break;
      tc_fence_after();
      {
        float x[32];
        tmem_ld32(xq + half * 32, x);
        tmem_wait_ld();
#pragma unroll
        for (int i4 = 0; i4 < 32; i4 += 4) {
          const float4 b4 = *reinterpret_cast<const float4*>(gates + GATE_BETA + half * 32 + i4);
          const float4 e4 = *reinterpret_cast<const float4*>(gates + GATE_EG + half * 32 + i4);
          x[i4] = tf32_rn(fmaf(-b4.x * e4.x, x[i4], bv[i4]));
          x[i4 + 1] = tf32_rn(fmaf(-b4.y * e4.y, x[i4 + 1], bv[i4 + 1]));
          x[i4 + 2] = tf32_rn(fmaf(-b4.z * e4.z, x[i4 + 2], bv[i4 + 2]));
          x[i4 + 3] = tf32_rn(fmaf(-b4.w * e4.w, x[i4 + 3], bv[i4 + 3]));
        }
        tmem_st32(xq + half * 32, x);
        tmem_wait_st();
      }
      tc_fence_before();
      named_sync(1, kEpiThreads);
      if (leader) {
        mbar_arrive(&bars[B_R_READY]);
        mbar_arrive(&bars[B_V_EMPTY]);
      }

      // gamma S ([X|Y] has read S); the state update then accumulates onto it.
      {
        const float gamma = gates[GATE_GAMMA];
        for (int cc = 0; cc < 2; ++cc) {
          const int col = half * 64 + cc * 32;
          float sv[32];
          tmem_ld32(tq + TM_S + col, sv);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[i] *= gamma;
          tmem_st32(tq + TM_S + col, sv);
        }
      }

      // Delta' = Delta diag(e^(G_last - G)) as packed bf16 hi / lo over the
      // dead R (the state update's operand, on the chain), then Delta rounded
      // to tf32 in place (the O product's operand, off it).
      float dg[32];
      load_gate32(gates + GATE_DG + half * 32, dg);
      ok = mbar_wait(&bars[B_D_DONE], par, wait_ns);
      if (!ok) record_error(&abort_flag);
      if (named_sync_or(1, kEpiThreads, !ok)) break;
      tc_fence_after();
      {
        float x[32];
        tmem_ld32(tq + TM_D + 64 * cb + half * 32, x);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) dg[i] *= x[i];
        uint32_t hi[16], lo[16];
        split32_packed(dg, hi, lo);
        tmem_st16(xq + half * 16, hi);
        tmem_st16(xq + 32 + half * 16, lo);
        tmem_wait_st();
        tc_fence_before();
        named_sync(1, kEpiThreads);
        if (leader) mbar_arrive(&bars[B_DD_READY]);
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = tf32_rn(x[i]);
        tmem_st32(tq + TM_D + 64 * cb + half * 32, x);
        tmem_wait_st();
      }
      tc_fence_before();
      named_sync(1, kEpiThreads);
      if (leader) mbar_arrive(&bars[B_DR_READY]);
    }

    // Final state (or the initial one for an empty sequence) -> state_out.
    bool ok = !abort_flag && (nch == 0 || mbar_wait(&bars[B_U_DONE], (uint32_t)((nch - 1) & 1), wait_ns));
    if (!ok && !abort_flag) record_error(&abort_flag);
    if (!named_sync_or(1, kEpiThreads, !ok) && chain_out) {
      tc_fence_after();
      float* orow = chain_out + (size_t)dv * DH;
      for (int cc = 0; cc < 2; ++cc) {
        const int col = half * 64 + cc * 32;
        float sv[32];
        tmem_ld32(tq + TM_S + col, sv);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(orow + col + i) = make_float4(sv[i], sv[i + 1], sv[i + 2], sv[i + 3]);
      }
    }
  } else if (warp < 14) {
    // ------------------------------------------------------------- output
    const int e = tid - 320;                  // 0..127 (warps 10-13)
    const int q = warp & 3;                   // TMEM lane quarter of this warp
    const int dv = q * 32 + lane;             // output row (value dim)
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    const bool leader = e == 0;
    unsigned char* sm = base;
    const int g8 = (e & 15) * 8;  // gated output: the 8 dv of this lane
    float nw[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) nw[j] = p.gated ? p.norm_w[g8 + j] : 0.f;
    const size_t ostride = (size_t)(GATHER ? p.out_hv : p.hv) * DH;
    // z of chunk c lands in its tile while chunk c - 1's output is formed:
    // the leader requests it as soon as the norm of chunk c - 1 has read the
    // tile (z of chunk 0 at once).
    const bool zload = p.gated && !(flags & kChainNoOut);
    int64_t n_z = 0;  // z tiles requested
    if (zload && leader && nch > 0) {
      mbar_arrive_expect_tx(&bars[B_Z_FULL], kBTile);
      tma_load_3d(sm + OFF_Z, &zmap, &bars[B_Z_FULL], 0, h, (int)start);
      n_z = 1;
    }
    for (int64_t c = 0; c < nch; ++c) {
      const int64_t t0 = start + c * CH;
      const int n = (int)(end - t0 < CH ? end - t0 : CH);
      const uint32_t cb = (uint32_t)(c & 1);
      // y = Y + O of this chunk (e^G is in Q~): all 64 tokens of row dv.
      bool ok = mbar_wait(&bars[B_OU_DONE0 + cb], (uint32_t)((c >> 1) & 1), wait_ns);
      if (!ok) record_error(&abort_flag);
      if (named_sync_or(2, kOutThreads, !ok)) break;
      tc_fence_after();
      float y[64];
      tmem_ld32(tq + TM_XY + 128 * cb + 64, *reinterpret_cast<float(*)[32]>(y));
      tmem_ld32(tq + TM_XY + 128 * cb + 96, *reinterpret_cast<float(*)[32]>(y + 32));
      tmem_wait_ld();
      if (leader) bulk_wait_group_read0();  // the previous tile store has left the staging buffer
      tc_fence_before();
      named_sync(2, kOutThreads);
      if (leader) mbar_arrive(&bars[B_Y_FREE0 + cb]);
      if (flags & kChainNoOut) continue;  // a transition chain: only its final state is wanted
      if (!p.gated) {
        if (n == CH) {
          // Whole chunk: stage [t][dv] in shared memory, one TMA tensor store.
          if (p.out_dtype == GDN_BF16) {
            unsigned short* st16 = reinterpret_cast<unsigned short*>(sm + OFF_OSTAGE);
#pragma unroll
            for (int i = 0; i < 64; i += 2) {
              const uint32_t w2 = cvt_bf16x2(y[i], y[i + 1]);
              st16[i * DH + dv] = (unsigned short)(w2 & 0xFFFFu);
              st16[(i + 1) * DH + dv] = (unsigned short)(w2 >> 16);
            }
          } else {
            float* st = reinterpret_cast<float*>(sm + OFF_OSTAGE);
#pragma unroll
            for (int i = 0; i < 64; ++i) st[i * DH + dv] = y[i];
          }
          fence_async_smem();
          named_sync(2, kOutThreads);
          if (leader) {
            tma_store_3d(&omap, sm + OFF_OSTAGE, 0, GATHER ? p.head0 + h : h, (int)t0);
            bulk_commit_group();
          }
          if (GATHER) copy_tile_to_peers(p, sm + OFF_OSTAGE, t0, CH, h, e);
        } else if (!GATHER) {  // ragged last chunk: plain stores of the valid rows
          if (p.out_dtype == GDN_BF16) {
            __nv_bfloat16* op = static_cast<__nv_bfloat16*>(p.out) + ((size_t)t0 * p.hv + h) * DH + dv;
#pragma unroll
            for (int i = 0; i < 64; ++i)
              if (i < n) op[i * ostride] = __float2bfloat16_rn(y[i]);
          } else {
            float* op = static_cast<float*>(p.out) + ((size_t)t0 * p.hv + h) * DH + dv;
#pragma unroll
            for (int i = 0; i < 64; ++i)
              if (i < n) op[i * ostride] = y[i];
          }
        } else {  // the same, here and at every peer
          const size_t obase = ((size_t)t0 * p.out_hv + p.head0 + h) * DH + dv;
          for (int j = -1; j < p.n_peers; ++j) {
            void* dst = j < 0 ? p.out : p.peer_out[j];
            if (p.out_dtype == GDN_BF16) {
              __nv_bfloat16* op = static_cast<__nv_bfloat16*>(dst) + obase;
#pragma unroll
              for (int i = 0; i < 64; ++i)
                if (i < n) op[i * ostride] = __float2bfloat16_rn(y[i]);
            } else {
              float* op = static_cast<float*>(dst) + obase;
#pragma unroll
              for (int i = 0; i < 64; ++i)
                if (i < n) op[i * ostride] = y[i];
            }
          }
        }
        continue;
      }
      // Fused-block output: y rounded to bf16 is staged [t][dv]; then the 16
      // lanes of a token (8 dv each) reduce its row, gate it with z (from its
      // tile) and overwrite it in place: out = silu(z) * rms_norm(y, w, eps).
      __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(sm + OFF_OSTAGE);
      unsigned short* st16 = reinterpret_cast<unsigned short*>(st);
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        const uint32_t w2 = cvt_bf16x2(y[i], y[i + 1]);
        st16[i * DH + dv] = (unsigned short)(w2 & 0xFFFFu);
        st16[(i + 1) * DH + dv] = (unsigned short)(w2 >> 16);
      }
      ok = mbar_wait(&bars[B_Z_FULL], (uint32_t)(c & 1), wait_ns);
      if (!ok) record_error(&abort_flag);
      if (named_sync_or(2, kOutThreads, !ok)) break;  // every row is staged, z has landed
      const __nv_bfloat16* zt = reinterpret_cast<const __nv_bfloat16*>(sm + OFF_Z);
      // The 8 items four at a time, phase by phase, so that the shuffle and
      // special-function latencies overlap.
#pragma unroll
      for (int i0 = 0; i0 < 8; i0 += 4) {
        uint4 yu[4], zu[4];
        float ss[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          yu[k] = *reinterpret_cast<const uint4*>(st + ((e >> 4) + 8 * (i0 + k)) * DH + g8);
          zu[k] = *reinterpret_cast<const uint4*>(zt + ((e >> 4) + 8 * (i0 + k)) * DH + g8);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t yw[4] = {yu[k].x, yu[k].y, yu[k].z, yu[k].w};
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float y0 = bf16_lo_f(yw[j]), y1 = bf16_hi_f(yw[j]);
            acc = fmaf(y0, y0, acc);
            acc = fmaf(y1, y1, acc);
          }
          ss[k] = acc;
        }
#pragma unroll
        for (int off = 8; off >= 1; off >>= 1)
#pragma unroll
          for (int k = 0; k < 4; ++k) ss[k] += __shfl_xor_sync(0xffffffffu, ss[k], off);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int tt = (e >> 4) + 8 * (i0 + k);
          const float inv = rsqrtf(ss[k] * (1.f / DH) + p.norm_eps);
          const uint32_t yw[4] = {yu[k].x, yu[k].y, yu[k].z, yu[k].w};
          const uint32_t zw[4] = {zu[k].x, zu[k].y, zu[k].z, zu[k].w};
          uint32_t ow[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float n0 = bf16_lo_f(yw[j]) * inv * nw[2 * j], n1 = bf16_hi_f(yw[j]) * inv * nw[2 * j + 1];
            round2_bf16(n0, n1);
            ow[j] = pack_bf16(silu_fast(bf16_lo_f(zw[j])) * n0, silu_fast(bf16_hi_f(zw[j])) * n1);
          }
          *reinterpret_cast<uint4*>(st + tt * DH + g8) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        }
      }
      fence_async_smem();
      named_sync(2, kOutThreads);  // every thread is done with z (and with the staged rows)
      if (leader && c + 1 < nch) {  // z of the next chunk into the tile just read
        mbar_arrive_expect_tx(&bars[B_Z_FULL], kBTile);
        tma_load_3d(sm + OFF_Z, &zmap, &bars[B_Z_FULL], 0, h, (int)(t0 + CH));
        n_z = c + 2;
      }
      if (n == CH) {
        if (leader) {
          tma_store_3d(&omap, sm + OFF_OSTAGE, 0, h, (int)t0);
          bulk_commit_group();
        }
      } else {  // ragged last chunk: the valid rows, 16 bytes per lane
        __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(p.out) + ((size_t)t0 * p.hv + h) * DH + g8;
        for (int it = 0; it < 8; ++it) {
          const int tt = (e >> 4) + 8 * it;
          if (tt < n) *reinterpret_cast<uint4*>(ob + (size_t)tt * ostride) = *reinterpret_cast<const uint4*>(st + tt * DH + g8);
        }
      }
    }
    if (leader) bulk_wait_group0();  // every output tile has reached global memory
    if (GATHER) __threadfence_system();  // the peer stores are visible beyond this GPU
    // After an abort, let the last z load in flight land (bounded) before the
    // CTA releases its shared memory (tile i completes phase i & 1).
    if (leader && n_z > 0) mbar_wait(&bars[B_Z_FULL], (uint32_t)((n_z - 1) & 1), wait_ns);
  } else {
    // ------------------------------------------------- bf16 -> tf32 operand tile
    // [K ; Q~]_c into the fp32 tile once [X|Y]_(c-1) has read it: K_c from its
    // bf16 tile (rows 0-63), Q~_c = diag(e^G) Q_c (rows 64-127).
    const int e = tid - 448;                  // 0..127 (warps 14-17)
    const bool leader = e == 0;
    for (int64_t c = 0; c < nch; ++c) {
      const int bb = (int)(c & 1);
      bool ok = !abort_flag && mbar_wait(&bars[B_K_FULL0 + bb], (uint32_t)((c >> 1) & 1), wait_ns) &&
                mbar_wait(&bars[B_Q_FULL], (uint32_t)(c & 1), wait_ns) &&
                (c == 0 || mbar_wait(&bars[B_X_DONE], (uint32_t)((c - 1) & 1), wait_ns));
      if (!ok && !abort_flag) record_error(&abort_flag);
      if (named_sync_or(3, kCvtThreads, !ok)) break;
      widen_tile(base + OFF_KB + bb * kBTile, base + OFF_KQ, 0, nullptr, e);
      widen_tile(base + OFF_QB, base + OFF_KQ, 64,
                 reinterpret_cast<const float*>(base + OFF_GATES + bb * kGateBytes) + GATE_EG, e);
      fence_async_smem();
      named_sync(3, kCvtThreads);
      if (leader) {
        mbar_arrive(&bars[B_Q_EMPTY]);
        mbar_arrive(&bars[B_KQ_READY]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

// 3-D map over a [N, H, 128] bf16 tensor with element strides (st, sh, 1);
// box {box_x, 1, 64}.
bool make_map(CUtensorMap* map, const void* ptr, int64_t n_tokens, int heads, int64_t st, int64_t sh, int box_x,
              bool swizzle) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  std::memset(map, 0, sizeof(*map));
  cuuint64_t dims[3] = {(cuuint64_t)DH, (cuuint64_t)heads, (cuuint64_t)n_tokens};
  cuuint64_t strides[2] = {(cuuint64_t)sh * 2, (cuuint64_t)st * 2};
  cuuint32_t box[3] = {(cuuint32_t)box_x, 1, (cuuint32_t)CH};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D map over the contiguous output [N, Hv, 128] (fp32 or bf16), box {128, 1, 64}.
bool make_out_map(CUtensorMap* map, void* ptr, int64_t n_tokens, int heads, gdn_dtype dt) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  std::memset(map, 0, sizeof(*map));
  const cuuint64_t es = dt == GDN_BF16 ? 2 : 4;
  cuuint64_t dims[3] = {(cuuint64_t)DH, (cuuint64_t)heads, (cuuint64_t)n_tokens};
  cuuint64_t strides[2] = {DH * es, (cuuint64_t)heads * DH * es};
  cuuint32_t box[3] = {(cuuint32_t)DH, 1, (cuuint32_t)CH};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt == GDN_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, ptr,
                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// ---------------------------------------------------------------------------
// One long sequence in segments.  The chunk chain maps a segment's start
// state affinely, S_end = S_start M + U: M (Dk x Dk) is the same recurrence
// run with V = 0 from the identity, U its end state from zero.  With P
// segments, phase 1 runs segment 0 for real (its outputs and end state are
// final) together with U_i and M_i of segments 1..P-2, all in one launch;
// phase 2 chains S_start(i+1) = S_start(i) M_i + U_i (fp32, per head); phase 3
// reruns segments 1..P-1 from their start states.  Every chain is shorter by
// about P, and phase 1's 1 + 2(P-2) chains per head still fit one wave.
// ---------------------------------------------------------------------------
constexpr int kMaxSegs = 8;
constexpr int kSmCount = 148;      // B200: phase-1 chains are kept within one wave of CTAs
constexpr int kMinSegChunks = 8;   // shorter segments cost more than they save

struct SegCu {
  int64_t cu[kMaxSegs + 1];
};

__global__ void seg_setup_kernel(const SegCu c, int n, int64_t* cu) {
  if (threadIdx.x <= n) cu[threadIdx.x] = c.cu[threadIdx.x];
}

// Every start state of a segmented sequence in one launch: W_j = W_(j-1) M_j +
// U_j for j = 1 .. n and every head (128 x 128 fp32 each; W_j holds U_j on
// entry).  Grid (Hv, 4): 32 rows of one head per CTA.  A row block of W_j
// depends only on the same rows of W_(j-1), so each CTA walks j on its own:
// its rows of W_(j-1) stay in shared memory from the step before, M_j (64 KB)
// is staged per step with every load in flight at once; thread = 2 rows x 8
// columns.
constexpr size_t kCombineSmem = (size_t)(DH + 32) * DH * sizeof(float);
__global__ void __launch_bounds__(256) state_combine_kernel(float* W, const float* Mt, int n, size_t hstate) {
  extern __shared__ __align__(16) float csm[];
  float* sm = csm;            // [128][128] M_j
  float* sa = csm + DH * DH;  // [32][128] rows of W_(j-1)
  const int tid = threadIdx.x, r = (tid >> 4) * 2, c0 = (tid & 15) * 8;
  const size_t head = (size_t)blockIdx.x * DH * DH;
  const int r0 = blockIdx.y * 32;
  {
    const float4* A = reinterpret_cast<const float4*>(W + head + (size_t)r0 * DH);
#pragma unroll 4
    for (int i = tid; i < 32 * DH / 4; i += 256) reinterpret_cast<float4*>(sa)[i] = A[i];
  }
  for (int j = 1; j <= n; ++j) {
    const float4* Mh = reinterpret_cast<const float4*>(Mt + (size_t)(j - 1) * hstate + head);
#pragma unroll 4
    for (int i = tid; i < DH * DH / 4; i += 256) reinterpret_cast<float4*>(sm)[i] = Mh[i];
    float* C = W + (size_t)j * hstate + head + (size_t)(r0 + r) * DH + c0;
    float acc[2][8];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const float4 x0 = *reinterpret_cast<const float4*>(C + rr * DH);
      const float4 x1 = *reinterpret_cast<const float4*>(C + rr * DH + 4);
      acc[rr][0] = x0.x; acc[rr][1] = x0.y; acc[rr][2] = x0.z; acc[rr][3] = x0.w;
      acc[rr][4] = x1.x; acc[rr][5] = x1.y; acc[rr][6] = x1.z; acc[rr][7] = x1.w;
    }
    __syncthreads();  // M_j and the rows of W_(j-1) are staged
#pragma unroll 4
    for (int k = 0; k < DH; ++k) {
      const float a0 = sa[r * DH + k], a1 = sa[(r + 1) * DH + k];
      const float4 m0 = *reinterpret_cast<const float4*>(sm + k * DH + c0);
      const float4 m1 = *reinterpret_cast<const float4*>(sm + k * DH + c0 + 4);
      const float mv[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        acc[0][jj] = fmaf(a0, mv[jj], acc[0][jj]);
        acc[1][jj] = fmaf(a1, mv[jj], acc[1][jj]);
      }
    }
    __syncthreads();  // every thread is done with M_j and with W_(j-1)
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const float4 lo = make_float4(acc[rr][0], acc[rr][1], acc[rr][2], acc[rr][3]);
      const float4 hi = make_float4(acc[rr][4], acc[rr][5], acc[rr][6], acc[rr][7]);
      *reinterpret_cast<float4*>(C + rr * DH) = lo;
      *reinterpret_cast<float4*>(C + rr * DH + 4) = hi;
      *reinterpret_cast<float4*>(sa + (r + rr) * DH + c0) = lo;
      *reinterpret_cast<float4*>(sa + (r + rr) * DH + c0 + 4) = hi;
    }
  }
}

// A second stream (and its fork / join events) per device, made on first use.
// Every caller on a device shares them, so a caller holds `lock` from the
// fork record to its wait on the join: another caller's record of either
// event cannot then land between this caller's record and its wait (the
// events are not reused until both waits have been enqueued, and a wait
// enqueues the event's state at the time of the call).
struct SideStream {
  cudaStream_t stream;
  cudaEvent_t fork, join;
  std::mutex lock;
  bool made;
};
SideStream* side_stream() {
  static SideStream streams[kMaxDevices];
  static std::mutex create;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> g(create);
  SideStream& x = streams[dev];
  if (!x.made) {
    int lo = 0, hi = 0;  // numerically greatest = lowest priority
    if (cudaDeviceGetStreamPriorityRange(&lo, &hi) != cudaSuccess ||
        cudaStreamCreateWithPriority(&x.stream, cudaStreamNonBlocking, lo) != cudaSuccess ||
        cudaEventCreateWithFlags(&x.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&x.join, cudaEventDisableTiming) != cudaSuccess)
      return nullptr;
    x.made = true;
  }
  return &x;
}

// Segments for one scan (1 = run it whole): only a single dense sequence whose
// heads leave most of the GPU idle is split.
int seg_count(const ScanParams& p) {
  if (p.n_seqs != 1 || p.cu_seqlens) return 1;
  const int64_t nch = (p.n_tokens + CH - 1) / CH;
  int P = 1;
  for (int q = 3; q <= kMaxSegs; ++q) {
    if ((int64_t)p.hv * (2 * q - 3) > kSmCount || nch < (int64_t)kMinSegChunks * q) break;
    P = q;
  }
  return P;
}

struct SegLayout {
  size_t recs, cu, w, m, total;
};

SegLayout seg_layout(const ScanParams& p, int P) {
  SegLayout L;
  const size_t state = (size_t)p.hv * DH * DH * sizeof(float);
  const int64_t nseq = P > 1 ? P : p.n_seqs;
  L.recs = (size_t)((p.n_tokens + CH - 1) / CH + nseq) * p.hv * kRecBytes;
  L.cu = (L.recs + 255) & ~(size_t)255;
  L.w = L.cu + (P > 1 ? 256 : 0);
  L.m = L.w + (P > 1 ? (size_t)(P - 1) * state : 0);
  L.total = L.m + (P > 1 ? (size_t)(P - 2) * state : 0);
  return L;
}

// The scan instance for these parameters (the gathered one only when asked).
using ScanKernel = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, ChunkParams);
ScanKernel scan_kernel(const ChunkParams& p) {
  const bool gather = p.n_peers > 0 || p.head0 != 0 || p.out_hv != p.hv;
  return gather ? chunk_scan_kernel<true> : chunk_scan_kernel<false>;
}

bool aligned_elems(int64_t s) { return s >= 0 && s % 8 == 0; }
bool aligned_ptr16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

bool chunked_supported(const ScanParams& p) {
  return p.qkv_dtype == GDN_BF16 && p.dk == DH && p.dv == DH && p.hv % p.hk == 0 && aligned_elems(p.q_st) &&
         aligned_elems(p.q_sh) && aligned_elems(p.k_st) && aligned_elems(p.k_sh) && aligned_elems(p.v_st) &&
         aligned_elems(p.v_sh) && p.n_tokens < (int64_t)1 << 31 && tensor_map_encoder() != nullptr;
}

size_t chunked_workspace_bytes(const ScanParams& p) { return seg_layout(p, seg_count(p)).total; }

cudaError_t launch_chunked_scan(const ScanParams& sp, cudaStream_t s) {
  if (!aligned_ptr16(sp.q) || !aligned_ptr16(sp.k) || !aligned_ptr16(sp.v) || !aligned_ptr16(sp.workspace))
    return cudaErrorMisalignedAddress;
  CUtensorMap qmap, kmap, vmap, omap, zmap;
  const int64_t N = sp.n_tokens;
  const bool gated = sp.z != nullptr;
  if (gated && (sp.out_dtype != GDN_BF16 || !aligned_ptr16(sp.z) || !aligned_elems(sp.z_st) || !sp.norm_w))
    return cudaErrorInvalidValue;
  std::memset(&zmap, 0, sizeof(zmap));
  if (N > 0) {
    if (!make_map(&qmap, sp.q, N, sp.hk, sp.q_st, sp.q_sh, 64, true) ||
        !make_map(&kmap, sp.k, N, sp.hk, sp.k_st, sp.k_sh, 64, true) ||
        !make_map(&vmap, sp.v, N, sp.hv, sp.v_st, sp.v_sh, 128, false) ||
        !make_out_map(&omap, sp.out, N, sp.out_hv > 0 ? sp.out_hv : sp.hv, sp.out_dtype) ||
        (gated && !make_map(&zmap, sp.z, N, sp.hv, sp.z_st, DH, 128, false)))
      return cudaErrorInvalidValue;
  } else {
    std::memset(&qmap, 0, sizeof(qmap));
    kmap = vmap = omap = qmap;
  }
  ChunkParams p;
  p.n_tokens = N;
  p.n_seqs = sp.n_seqs;
  p.cu = sp.cu_seqlens;
  p.hk = sp.hk;
  p.hv = sp.hv;
  p.g = sp.g;
  p.beta = sp.beta;
  p.g_st = sp.g_st;
  p.beta_st = sp.beta_st;
  p.gate_dtype = sp.gate_dtype;
  p.gate_kind = sp.gate_kind;
  p.state_in = sp.state_in;
  p.state_out = sp.state_out;
  p.out = sp.out;
  p.out_dtype = sp.out_dtype;
  p.ws = static_cast<unsigned char*>(sp.workspace);
  p.rec0 = 0;
  p.gated = gated ? 1 : 0;
  p.norm_w = sp.norm_w;
  p.norm_eps = sp.norm_eps;
  p.z = static_cast<const __nv_bfloat16*>(sp.z);
  p.z_st = sp.z_st;
  p.out_hv = sp.out_hv > 0 ? sp.out_hv : sp.hv;
  p.head0 = sp.head0;
  p.n_peers = sp.n_peers;
  for (int j = 0; j < GDN_MAX_GATHER_PEERS; ++j) p.peer_out[j] = j < sp.n_peers ? sp.peer_out[j] : nullptr;
  if (gated && (p.out_hv != sp.hv || p.head0 || p.n_peers)) return cudaErrorInvalidValue;  // the fused block is not gathered

  {
    static DeviceFlags prep_attr, scan_attr, gather_attr, comb_attr;
    cudaError_t e = ensure_smem_attr(chunk_prep_kernel, kPrepSmem, prep_attr);
    if (e != cudaSuccess) return e;
    e = ensure_smem_attr(chunk_scan_kernel<false>, kScanSmem, scan_attr);
    if (e != cudaSuccess) return e;
    e = ensure_smem_attr(chunk_scan_kernel<true>, kScanSmem, gather_attr);
    if (e != cudaSuccess) return e;
    e = ensure_smem_attr(state_combine_kernel, kCombineSmem, comb_attr);
    if (e != cudaSuccess) return e;
  }
  p.n_chains = 0;
  const int P = seg_count(sp);
  if (P > 1) {
    // Segment boundaries on chunk multiples, segment 0 first.
    const SegLayout L = seg_layout(sp, P);
    const int64_t nch = (N + CH - 1) / CH;
    SegCu sc;
    for (int i = 0; i <= P; ++i) sc.cu[i] = std::min<int64_t>(N, (nch * i / P) * CH);
    int64_t* cu_dev = reinterpret_cast<int64_t*>(p.ws + L.cu);
    seg_setup_kernel<<<1, 32, 0, s>>>(sc, P, cu_dev);
    p.cu = cu_dev;
    p.n_seqs = P;
  }
  if (P <= 1) {
    const int64_t slots = (N + CH - 1) / CH + p.n_seqs;
    if (N > 0 && slots > 0) {
      if (slots > 0x7fffffffLL || sp.hv > 65535) return cudaErrorInvalidConfiguration;
      chunk_prep_kernel<<<dim3((unsigned)slots, (unsigned)sp.hv), 128, kPrepSmem, s>>>(qmap, kmap, p);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return e;
    }
    const int64_t ctas = sp.n_seqs * sp.hv;
    if (ctas > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    scan_kernel(p)<<<(unsigned)ctas, kScanThreads, kScanSmem, s>>>(qmap, kmap, vmap, omap, zmap, p);
    return cudaGetLastError();
  }
  // Chunk records: segments 0..P-2 before phase 1; the last segment's (needed
  // only by phase 3) on a low-priority side stream that starts with phase 1,
  // on the SMs phase 1 leaves free.
  SideStream* side = side_stream();
  if (!side) return cudaErrorNotReady;
  std::lock_guard<std::mutex> side_guard(side->lock);  // fork record .. join wait
  const int64_t nch_all = (N + CH - 1) / CH;
  const int64_t last0 = (nch_all * (P - 1) / P);  // first chunk of the last segment
  {
    ChunkParams pf = p;
    pf.n_seqs = P - 1;
    chunk_prep_kernel<<<dim3((unsigned)(last0 + P - 1), (unsigned)sp.hv), 128, kPrepSmem, s>>>(qmap, kmap, pf);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  e = cudaEventRecord(side->fork, s);
  if (e != cudaSuccess) return e;
  e = cudaStreamWaitEvent(side->stream, side->fork, 0);
  if (e != cudaSuccess) return e;
  {
    ChunkParams pl = p;
    pl.cu = p.cu + (P - 1);
    pl.n_seqs = 1;
    pl.rec0 = last0;  // records are numbered by chunk over the segments in order
    chunk_prep_kernel<<<dim3((unsigned)(nch_all - last0 + 1), (unsigned)sp.hv), 128, kPrepSmem, side->stream>>>(
        qmap, kmap, pl);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  e = cudaEventRecord(side->join, side->stream);
  if (e != cudaSuccess) return e;
  const SegLayout L = seg_layout(sp, P);
  const size_t hstate = (size_t)sp.hv * DH * DH;
  float* W = reinterpret_cast<float*>(p.ws + L.w);  // end states of segments 0..P-2, then their start states
  float* Mt = reinterpret_cast<float*>(p.ws + L.m); // transitions of segments 1..P-2
  // phase 1: segment 0 for real; U_i and M_i of segments 1..P-2
  ChunkParams p1 = p;
  p1.n_chains = 1 + 2 * (P - 2);
  p1.chains[0] = {0, sp.state_in, W, 0};
  for (int i = 1; i <= P - 2; ++i) {
    p1.chains[i] = {i, nullptr, W + i * hstate, kChainNoOut};
    p1.chains[P - 2 + i] = {i, nullptr, Mt + (i - 1) * hstate, kChainIdentity | kChainZeroV | kChainNoOut};
  }
  scan_kernel(p1)<<<(unsigned)(p1.n_chains * sp.hv), kScanThreads, kScanSmem, s>>>(qmap, kmap, vmap, omap, zmap, p1);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // phase 2: start states, W[j] = W[j-1] M_j + U_j for j = 1 .. P-2, one launch
  if (P > 2) {
    state_combine_kernel<<<dim3((unsigned)sp.hv, DH / 32), 256, kCombineSmem, s>>>(W, Mt, P - 2, hstate);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  // phase 3: segments 1..P-1 from their start states; the last one's end state is the result
  e = cudaStreamWaitEvent(s, side->join, 0);
  if (e != cudaSuccess) return e;
  ChunkParams p3 = p;
  p3.n_chains = P - 1;
  for (int i = 1; i <= P - 1; ++i) p3.chains[i - 1] = {i, W + (i - 1) * hstate, i == P - 1 ? sp.state_out : nullptr, 0};
  scan_kernel(p3)<<<(unsigned)(p3.n_chains * sp.hv), kScanThreads, kScanSmem, s>>>(qmap, kmap, vmap, omap, zmap, p3);
  return cudaGetLastError();
}

cudaError_t set_test_hooks(unsigned long long wait_ns, int fault) {
  if (!wait_ns) wait_ns = kDefaultWaitNs;
  cudaError_t e = cudaMemcpyToSymbol(g_wait_limit_ns, &wait_ns, sizeof(wait_ns));
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_test_fault, &fault, sizeof(fault));
}

cudaError_t read_test_hooks(unsigned long long* wait_ns, int* fault) {
  cudaError_t e = cudaMemcpyFromSymbol(wait_ns, g_wait_limit_ns, sizeof(*wait_ns));
  if (e != cudaSuccess) return e;
  return cudaMemcpyFromSymbol(fault, g_test_fault, sizeof(*fault));
}

cudaError_t read_and_clear_device_error(unsigned* code) {
  cudaError_t e = cudaMemcpyFromSymbol(code, g_device_error, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  if (*code) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(unsigned));
  }
  return e;
}

}  // namespace gdn
