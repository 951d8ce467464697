// Linear projection with affine-quantized weights on the sm_100a tensor
// cores: out = x W^T, W[n, k] = scale[n, k / gs] * q[n, k] + bias[n, k / gs]
// (the reference's quantized_linear, model/moe_block.py:23-50, which calls
// mx.quantized_matmul in its affine mode).
//
// One CTA per 128 x 256 output tile (tokens x output features), looping over
// K in blocks of 64:
//   warp 0     TMA: the x tile (128 x 64 bf16, 128-byte swizzle) and the
//              packed weight rows (256 x 64 values) into a 3-stage ring;
//   warps 2-9  dequantization: thread r expands row r of the weight block
//              into bf16, in the 128-byte-swizzled K-major operand layout
//              (2-stage ring), then, after the last block, the epilogue;
//   warp 1     one tcgen05.mma (M = 128, N = 256, K = 16) per 16 of K into a
//              128 x 256 fp32 accumulator in TMEM.
// 4-bit values become bf16 pairs with the magic-number method (OR the nibble
// into the mantissa of 128.0, subtract 128: Kim et al., "Who Says Elephants
// Can't Run", 2022), then one bf16x2 FMA with the group's scale and bias: a
// single rounding of s * q + b to bf16.  8-bit values go through float32
// (OR into the mantissa of 2^23) and one FMA, then a pairwise bf16 rounding.
// The epilogue stages the tile as four 128 x 64 bf16 sub-tiles (128-byte
// swizzle) and writes them with TMA stores; the TMA loads zero-fill, and the
// stores clip, the parts of edge tiles outside x and out.
//
// Every wait is bounded (2 s); on a timeout the kernel records an error for
// gdn_check_device_errors, lets its own copies and MMAs land (bounded), frees
// its TMEM and returns.
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <cstring>

#include "gdn_common.cuh"
#include "gdn_sm100.cuh"

namespace gdn {

__device__ unsigned g_qlinear_error = 0;

namespace {

using namespace sm100;

constexpr int QBM = 128, QBN = 256, QBK = 64;
constexpr int kAStages = 3, kBStages = 2;
constexpr uint32_t kATile = QBM * QBK * 2;            // 16 KB
constexpr uint32_t kWTile = QBN * QBK;                // up to 8-bit: 16 KB
constexpr uint32_t kBTile = QBN * QBK * 2;            // 32 KB
constexpr uint32_t QOFF_A = 0;
constexpr uint32_t QOFF_W = QOFF_A + kAStages * kATile;
constexpr uint32_t QOFF_B = QOFF_W + kAStages * kWTile;  // also the output staging (4 x 16 KB)
constexpr uint32_t QSMEM_USED = QOFF_B + kBStages * kBTile;
constexpr size_t kQSmem = 1024 + QSMEM_USED;
constexpr int kDqThreads = 256;  // warps 2-9
constexpr uint64_t kQWaitNs = 2000000000ull;

struct QParams {
  int64_t m, n, k;
  const __nv_bfloat16* scales;
  const __nv_bfloat16* biases;
  int bits, gs;
};

enum QBar { Q_FULL0, Q_EMPTY0 = Q_FULL0 + kAStages, Q_BFULL0 = Q_EMPTY0 + kAStages, Q_BEMPTY0 = Q_BFULL0 + kBStages,
            Q_ACC = Q_BEMPTY0 + kBStages, Q_NBARS };

__device__ __forceinline__ void q_record(volatile int* abort_flag) {
  *abort_flag = 1;
  atomicOr(&g_qlinear_error, kErrTimeout);
}

// bf16x2 with the two values' bits in its halves, as a __nv_bfloat162.
__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t u) { return *reinterpret_cast<__nv_bfloat162*>(&u); }
__device__ __forceinline__ uint32_t as_u32(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }

// Eight 4-bit values of one word -> four bf16x2 words s * q + b.
__device__ __forceinline__ uint4 dequant_word4(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 b2) {
  const __nv_bfloat162 k128 = as_bf2(0x43004300u);  // (128.0, 128.0)
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t t = w >> (8 * i);
    const uint32_t p = (t & 0xFu) | ((t << 12) & 0xF0000u) | 0x43004300u;  // (128 + q_2i, 128 + q_2i+1)
    o[i] = as_u32(__hfma2(__hsub2(as_bf2(p), k128), s2, b2));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Four 8-bit values of each of two words -> four bf16x2 words s * q + b.
__device__ __forceinline__ uint4 dequant_words8(uint32_t w0, uint32_t w1, float s, float b) {
  uint32_t o[4];
  const uint32_t ws[2] = {w0, w1};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w = ws[i >> 1];
    const int sh = 16 * (i & 1);
    const float q0 = __uint_as_float(0x4B000000u | ((w >> sh) & 0xFFu)) - 8388608.f;
    const float q1 = __uint_as_float(0x4B000000u | ((w >> (sh + 8)) & 0xFFu)) - 8388608.f;
    o[i] = cvt_bf16x2(fmaf(s, q0, b), fmaf(s, q1, b));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void __launch_bounds__(320, 1) qlinear_kernel(const __grid_constant__ CUtensorMap amap,
                                                         const __grid_constant__ CUtensorMap wmap,
                                                         const __grid_constant__ CUtensorMap omap, const QParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bars[Q_NBARS];
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t n0 = (int64_t)blockIdx.x * QBN, m0 = (int64_t)blockIdx.y * QBM;
  const int nk = (int)(p.k / QBK);
  const uint32_t wbytes = (uint32_t)(QBK * p.bits / 8);  // packed bytes of one weight row per K-block
  const int wwords = QBK * p.bits / 32;

  if (tid == 0) {
    abort_flag = 0;
    for (int i = 0; i < Q_NBARS; ++i) {
      const bool empty = i >= Q_EMPTY0 && i < Q_EMPTY0 + kAStages;  // MMA commit + dequantizers
      mbar_init(&bars[i], empty ? 2 : 1);
    }
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base, QBN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&amap);
      prefetch_tensormap(&wmap);
      int issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kAStages;
        if (kb >= kAStages && !mbar_wait(&bars[Q_EMPTY0 + s], (uint32_t)((kb / kAStages - 1) & 1), kQWaitNs))
          q_record(&abort_flag);
        if (abort_flag) break;
        mbar_arrive_expect_tx(&bars[Q_FULL0 + s], kATile + wbytes * QBN);
        tma_load_2d(base + QOFF_A + s * kATile, &amap, &bars[Q_FULL0 + s], kb * QBK, (int)m0);
        tma_load_2d(base + QOFF_W + s * kWTile, &wmap, &bars[Q_FULL0 + s], kb * wwords, (int)n0);
        ++issued;
      }
      // After an abort, let this thread's copies land (bounded) before the
      // CTA releases its shared memory.
      if (abort_flag)
        for (int kb = issued - kAStages < 0 ? 0 : issued - kAStages; kb < issued; ++kb)
          mbar_wait(&bars[Q_FULL0 + kb % kAStages], (uint32_t)((kb / kAStages) & 1), kQWaitNs);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(QBM, QBN);
      int kb = 0;
      for (; kb < nk; ++kb) {
        const int s = kb % kAStages, sb = kb % kBStages;
        if (!mbar_wait(&bars[Q_FULL0 + s], (uint32_t)((kb / kAStages) & 1), kQWaitNs) ||
            !mbar_wait(&bars[Q_BFULL0 + sb], (uint32_t)((kb / kBStages) & 1), kQWaitNs)) {
          q_record(&abort_flag);
          break;
        }
        if (abort_flag) break;
        tc_fence_after();
        const uint32_t a = smem_u32(base + QOFF_A + s * kATile), b = smem_u32(base + QOFF_B + sb * kBTile);
#pragma unroll
        for (int ks = 0; ks < QBK / 16; ++ks)
          mma_bf16(tmem, sdesc_sw128(a + ks * 32), sdesc_sw128(b + ks * 32), idesc, kb > 0 || ks > 0);
        mma_commit(&bars[Q_EMPTY0 + s]);
        mma_commit(&bars[Q_BEMPTY0 + sb]);
      }
      // The accumulator is complete (or, after an abort, every MMA issued
      // has finished) when this commit's barrier completes.
      mma_commit(&bars[Q_ACC]);
      if (kb < nk) mbar_wait(&bars[Q_ACC], 0, kQWaitNs);
    }
  } else {
    // ------------------------------------------- dequantization, then epilogue
    const int r = tid - 64;  // weight row of the tile (0..255)
    const int64_t row = n0 + r;
    const bool live = row < p.n;
    const int64_t groups = p.k / p.gs;
    const __nv_bfloat16* srow = p.scales + (live ? row : 0) * groups;
    const __nv_bfloat16* brow = p.biases ? p.biases + (live ? row : 0) * groups : nullptr;
    const __nv_bfloat16 bzero = __float2bfloat16_rn(0.f);
    // (scale, bias) of this row's first and second half of a K-block, one block ahead.
    auto gate_of = [&](int kb, int hlf) -> int64_t { return ((int64_t)kb * QBK + hlf * 32) / p.gs; };
    __nv_bfloat16 s_nx[2], b_nx[2];
#pragma unroll
    for (int hlf = 0; hlf < 2; ++hlf) {
      s_nx[hlf] = live ? srow[gate_of(0, hlf)] : bzero;
      b_nx[hlf] = (live && brow) ? brow[gate_of(0, hlf)] : bzero;
    }
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kAStages, sb = kb % kBStages;
      const __nv_bfloat16 s_cur[2] = {s_nx[0], s_nx[1]}, b_cur[2] = {b_nx[0], b_nx[1]};
      if (kb + 1 < nk) {
#pragma unroll
        for (int hlf = 0; hlf < 2; ++hlf) {
          s_nx[hlf] = live ? srow[gate_of(kb + 1, hlf)] : bzero;
          b_nx[hlf] = (live && brow) ? brow[gate_of(kb + 1, hlf)] : bzero;
        }
      }
      ok = mbar_wait(&bars[Q_FULL0 + s], (uint32_t)((kb / kAStages) & 1), kQWaitNs) &&
           (kb < kBStages || mbar_wait(&bars[Q_BEMPTY0 + sb], (uint32_t)((kb / kBStages - 1) & 1), kQWaitNs));
      if (!ok) q_record(&abort_flag);
      if (named_sync_or(1, kDqThreads, !ok)) break;
      const unsigned char* wsrc = base + QOFF_W + s * kWTile + (size_t)r * wbytes;
      unsigned char* bdst = base + QOFF_B + sb * kBTile;
      if (p.bits == 4) {
        const uint4 w0 = reinterpret_cast<const uint4*>(wsrc)[0], w1 = reinterpret_cast<const uint4*>(wsrc)[1];
        const uint32_t wd[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const __nv_bfloat162 s2 = __bfloat162bfloat162(s_cur[c >> 2]), b2 = __bfloat162bfloat162(b_cur[c >> 2]);
          const uint4 v = live ? dequant_word4(wd[c], s2, b2) : make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(bdst + sw128_chunk(QBN, r, 0, c)) = v;
        }
      } else {
        const uint4* w4 = reinterpret_cast<const uint4*>(wsrc);
#pragma unroll
        for (int c2 = 0; c2 < 4; ++c2) {
          const uint4 w = w4[c2];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int c = 2 * c2 + hh;
            const float sv = __bfloat162float(s_cur[c >> 2]), bv = __bfloat162float(b_cur[c >> 2]);
            const uint4 v = live ? dequant_words8(hh ? w.z : w.x, hh ? w.w : w.y, sv, bv) : make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4*>(bdst + sw128_chunk(QBN, r, 0, c)) = v;
          }
        }
      }
      fence_async_smem();
      named_sync(1, kDqThreads);
      if (r == 0) {
        mbar_arrive(&bars[Q_BFULL0 + sb]);  // the operand is ready
        mbar_arrive(&bars[Q_EMPTY0 + s]);   // the packed weights are read
      }
    }

    // ------------------------------------------------------------ epilogue
    ok = !abort_flag && mbar_wait(&bars[Q_ACC], 0, kQWaitNs);
    if (!ok) q_record(&abort_flag);
    if (!named_sync_or(1, kDqThreads, !ok)) {
      tc_fence_after();
      const int q = warp & 3, half = (warp - 2) >> 2;  // TMEM lane quarter; columns 128 * half ..
      const int orow = q * 32 + lane;                  // output row of the tile
      const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int jj = 0; jj < 2; ++jj) {
        const int j = half * 2 + jj;  // 64-column sub-tile
        float v[64];
        tmem_ld32(tq + j * 64, *reinterpret_cast<float(*)[32]>(v));
        tmem_ld32(tq + j * 64 + 32, *reinterpret_cast<float(*)[32]>(v + 32));
        tmem_wait_ld();
        unsigned char* st = base + QOFF_B + j * (QBM * 128);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 o = make_uint4(cvt_bf16x2(v[8 * c], v[8 * c + 1]), cvt_bf16x2(v[8 * c + 2], v[8 * c + 3]),
                                     cvt_bf16x2(v[8 * c + 4], v[8 * c + 5]), cvt_bf16x2(v[8 * c + 6], v[8 * c + 7]));
          *reinterpret_cast<uint4*>(st + sw128_chunk(QBM, orow, 0, c)) = o;
        }
      }
      fence_async_smem();
      named_sync(1, kDqThreads);
      if (r == 0) {
        for (int j = 0; j < 4; ++j)
          if (n0 + 64 * j < p.n) tma_store_2d(&omap, base + QOFF_B + j * (QBM * 128), (int)(n0 + 64 * j), (int)m0);
        bulk_commit_group();
        bulk_wait_group_read0();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, QBN);
}

// Dense copy of the dequantized weights: thread per (row, word).
template <typename TO>
__global__ void dequant_kernel(const uint32_t* __restrict__ w, const QParams p, TO* __restrict__ dense) {
  const int64_t words_per_row = p.k * p.bits / 32;
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= p.n * words_per_row) return;
  const int64_t row = i / words_per_row, wi = i % words_per_row;
  const int per = 32 / p.bits;
  const uint32_t word = w[i];
  const uint32_t mask = (1u << p.bits) - 1u;
  for (int j = 0; j < per; ++j) {
    const int64_t kk = wi * per + j;
    const int64_t g = kk / p.gs;
    const float s = __bfloat162float(p.scales[row * (p.k / p.gs) + g]);
    const float b = p.biases ? __bfloat162float(p.biases[row * (p.k / p.gs) + g]) : 0.f;
    const float q = (float)((word >> (j * p.bits)) & mask);
    // the same single rounding to bf16 as the GEMM's operand
    const float v = __bfloat162float(__float2bfloat16_rn(fmaf(s, q, b)));
    dense[row * p.k + kk] = from_f<TO>(v);
  }
}

}  // namespace

namespace {

PFN_cuTensorMapEncodeTiled_v12000 q_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (PFN_cuTensorMapEncodeTiled_v12000) nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

// 2-D map: inner extent `cols`, `rows` rows of `row_bytes`, box {box_cols, box_rows}.
bool q_map(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt, int64_t cols, int64_t rows,
           int64_t row_bytes, int box_cols, int box_rows, bool swizzle) {
  auto enc = q_encoder();
  if (!enc) return false;
  std::memset(map, 0, sizeof(*map));
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  return enc(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

gdn_status q_check(const gdn_qlinear_args* a, QParams* p) {
  if (!a) return set_error(GDN_EINVAL, "args is NULL");
  if (a->m < 0 || a->n <= 0 || a->k <= 0) return set_error(GDN_EINVAL, "quantized_linear needs m >= 0, n > 0, k > 0");
  if (a->bits != 4 && a->bits != 8)
    return set_error(GDN_EUNSUPPORTED, "quantized_linear supports bits 4 and 8 (got %d)", a->bits);
  if (a->group_size != 32 && a->group_size != 64 && a->group_size != 128)
    return set_error(GDN_EUNSUPPORTED, "group_size must be 32, 64 or 128 (got %d)", a->group_size);
  if (a->k % 64 || a->k % a->group_size)
    return set_error(GDN_EUNSUPPORTED, "k (%lld) must be a multiple of 64 and of group_size", (long long)a->k);
  if (!a->w || !a->scales || (a->m > 0 && (!a->x || !a->out)))
    return set_error(GDN_EINVAL, "x, w, scales and out must be non-NULL");
  if (a->m > 0 && (a->x_stride_m < a->k || a->x_stride_m % 8 || a->out_stride_m < a->n || a->out_stride_m % 8))
    return set_error(GDN_EINVAL, "row strides must cover the rows and be multiples of 8 elements");
  if (!a16(a->w) || (a->m > 0 && (!a16(a->x) || !a16(a->out))))
    return set_error(GDN_EINVAL, "x, w and out must be 16-byte aligned");
  if (a->n > 0x7fffffffLL || a->m > 0x7fffffffLL || a->k > 0x7fffffffLL)
    return set_error(GDN_EUNSUPPORTED, "dimensions must be < 2^31");
  p->m = a->m;
  p->n = a->n;
  p->k = a->k;
  p->scales = static_cast<const __nv_bfloat16*>(a->scales);
  p->biases = static_cast<const __nv_bfloat16*>(a->biases);
  p->bits = a->bits;
  p->gs = a->group_size;
  return GDN_OK;
}

gdn_status q_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return GDN_OK;
  return set_error(GDN_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace

cudaError_t read_and_clear_qlinear_error(unsigned* code) {
  cudaError_t e = cudaMemcpyFromSymbol(code, g_qlinear_error, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  if (*code) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_qlinear_error, &zero, sizeof(unsigned));
  }
  return e;
}

}  // namespace gdn

extern "C" gdn_status gdn_quantized_linear(const gdn_qlinear_args* a, gdn_stream_t stream) {
  gdn::QParams p;
  gdn_status st = gdn::q_check(a, &p);
  if (st != GDN_OK || a->m == 0) return st;
  CUtensorMap amap, wmap, omap;
  const int64_t kw = a->k * a->bits / 32;  // words per weight row
  if (!gdn::q_map(&amap, a->x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a->k, a->m, a->x_stride_m * 2, 64, 128, true) ||
      !gdn::q_map(&wmap, a->w, CU_TENSOR_MAP_DATA_TYPE_UINT32, kw, a->n, kw * 4, 64 * a->bits / 32, 256, false) ||
      !gdn::q_map(&omap, a->out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a->n, a->m, a->out_stride_m * 2, 64, 128, true))
    return gdn::set_error(GDN_ECUDA, "quantized_linear: tensor map encoding failed");
  static bool attr = false;
  if (!attr) {
    st = gdn::q_cuda(cudaFuncSetAttribute(gdn::qlinear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)gdn::kQSmem),
                     "quantized_linear attribute");
    if (st != GDN_OK) return st;
    attr = true;
  }
  const dim3 grid((unsigned)((a->n + gdn::QBN - 1) / gdn::QBN), (unsigned)((a->m + gdn::QBM - 1) / gdn::QBM));
  if (grid.y > 65535) return gdn::set_error(GDN_EUNSUPPORTED, "m too large for one call (%lld)", (long long)a->m);
  gdn::qlinear_kernel<<<grid, 320, gdn::kQSmem, static_cast<cudaStream_t>(stream)>>>(amap, wmap, omap, p);
  return gdn::q_cuda(cudaGetLastError(), "quantized_linear launch");
}

extern "C" gdn_status gdn_dequantize(const gdn_qlinear_args* a, gdn_dtype out_dtype, void* dense,
                                     gdn_stream_t stream) {
  gdn::QParams p;
  gdn_qlinear_args b = *a;
  b.m = 0;  // no activations here
  gdn_status st = gdn::q_check(&b, &p);
  if (st != GDN_OK) return st;
  if (!dense) return gdn::set_error(GDN_EINVAL, "dense is NULL");
  if (out_dtype != GDN_F32 && out_dtype != GDN_BF16)
    return gdn::set_error(GDN_EUNSUPPORTED, "dequantize writes F32 or BF16");
  const int64_t total = a->n * (a->k * a->bits / 32);
  const unsigned blocks = (unsigned)((total + 255) / 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (out_dtype == GDN_F32)
    gdn::dequant_kernel<float><<<blocks, 256, 0, s>>>(a->w, p, static_cast<float*>(dense));
  else
    gdn::dequant_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(a->w, p, static_cast<__nv_bfloat16*>(dense));
  return gdn::q_cuda(cudaGetLastError(), "dequantize launch");
}
