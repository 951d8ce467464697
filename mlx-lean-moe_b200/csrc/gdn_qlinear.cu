// Linear projection with affine-quantized weights on the sm_100a tensor
// cores: out = x W^T, W[n, k] = scale[n, k / gs] * q[n, k] + bias[n, k / gs]
// (the reference's quantized_linear, model/moe_block.py:23-50, which calls
// mx.quantized_matmul in its affine mode).
//
// From 17 tokens on (qlinear_kernel): one CTA per 256 x 256 output tile
// (tokens x output features), looping over K in blocks of 64:
//   warp 0      TMA: the x tile (256 x 64 bf16, 128-byte swizzle) and the
//               packed weight rows (256 x 64 values) into a 3-stage ring,
//               and every 8 groups a tile of scales and biases (8 x 256 bf16)
//               into a 2-stage ring;
//   warps 2-17  dequantization: two threads per weight row (one per 32-value
//               half of the block) expand it into bf16 in the 128-byte-
//               swizzled K-major operand layout (2-stage ring); each warp
//               arrives for itself once its rows are written; after the
//               last block, the epilogue;
//   warp 1      two tcgen05.mma (M = 128, N = 256, K = 16) per 16 of K, one
//               per 128-row half of the tile, into two 128 x 256 fp32
//               accumulators in TMEM (all 512 columns).
// 4-bit values become bf16 pairs with the magic-number method (OR the nibble
// into the mantissa of 128.0, subtract 128: Kim et al., "Who Says Elephants
// Can't Run", 2022), then one bf16x2 FMA with the group's scale and bias: a
// single rounding of s * q + b to bf16.  8-bit values go through float32
// (a byte permute into the mantissa of 2^23) and one FMA, then a pairwise
// bf16 rounding.  The epilogue stages the tile as eight 128 x 64 bf16
// sub-tiles (128-byte swizzle) over the idle A and W rings and writes them
// with TMA stores; the TMA loads zero-fill, and the stores clip, the parts of
// edge tiles outside x, the weights and out.  Up to 16 tokens run the
// register-fed GEMV further down instead.
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

constexpr int QBM = 256, QBN = 256, QBK = 64;  // CTA tile: two 128-row accumulators share each B tile
constexpr int kAStages = 3, kBStages = 2;
constexpr uint32_t kATile = QBM * QBK * 2;            // 32 KB
constexpr uint32_t kWTile = QBN * QBK;                // up to 8-bit: 16 KB
constexpr uint32_t kBTile = QBN * QBK * 2;            // 32 KB
constexpr uint32_t kOutSub = 128 * 64 * 2;            // one 128 x 64 bf16 output sub-tile
constexpr uint32_t QOFF_A = 0;                        // A and W rings, then the output staging (8 sub-tiles)
constexpr uint32_t QOFF_W = QOFF_A + kAStages * kATile;
constexpr uint32_t QOFF_B = QOFF_W + kAStages * kWTile;
constexpr uint32_t kScTile = 8 * QBN * 2;                 // 8 groups x 256 rows of bf16 scales (or biases): 4 KB
constexpr uint32_t QOFF_SC = QOFF_B + kBStages * kBTile;  // 2 stages x (scales, biases)
constexpr uint32_t QSMEM_USED = QOFF_SC + 2 * 2 * kScTile;
static_assert(8 * kOutSub <= QOFF_B, "output staging overlaps the B ring");
constexpr size_t kQSmem = 1024 + QSMEM_USED;
constexpr int kDqThreads = 512;  // warps 2-17: two threads per weight row (one per 32-value half of a K-block)
constexpr int kDqWarps = kDqThreads / 32;
constexpr int kQThreads = 64 + kDqThreads;
constexpr uint64_t kQWaitNs = 2000000000ull;
constexpr int kScaleAhead = 8;  // K-blocks of scales and biases in flight per dequantizing thread

struct QParams {
  int64_t m, n, k;
  const __nv_bfloat16* scales;
  const __nv_bfloat16* biases;
  int bits, gs, gshift;  // gs == 1 << gshift
  int scale_tma;         // scales (and biases) arrive as TMA tiles of 8 groups x 256 rows
  int sshift;            // K-blocks per scale tile: 8 * gs / 64 == 1 << sshift
};

enum QBar { Q_FULL0, Q_EMPTY0 = Q_FULL0 + kAStages, Q_BFULL0 = Q_EMPTY0 + kAStages, Q_BEMPTY0 = Q_BFULL0 + kBStages,
            Q_ACC = Q_BEMPTY0 + kBStages, Q_SCFULL0, Q_SCEMPTY0 = Q_SCFULL0 + 2, Q_NBARS = Q_SCEMPTY0 + 2 };

__device__ __forceinline__ void q_record(volatile int* abort_flag) {
  *abort_flag = 1;
  atomicOr(&g_qlinear_error, kErrTimeout);
}

// bf16x2 with the two values' bits in its halves, as a __nv_bfloat162.
__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t u) { return *reinterpret_cast<__nv_bfloat162*>(&u); }
__device__ __forceinline__ uint32_t as_u32(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }

// Eight 4-bit values of one word -> four bf16x2 words s * q + b, in value
// order.  One AND-OR per pair puts nibbles j and j + 4 into the mantissas of
// (128.0, 128.0); a byte permute pairs them up as (2i, 2i + 1).
__device__ __forceinline__ uint4 dequant_word4(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 b2) {
  const uint32_t m = 0x000F000Fu, mag = 0x43004300u;
  const uint32_t p0 = (w & m) | mag, p1 = ((w >> 4) & m) | mag;  // (v0, v4), (v1, v5)
  const uint32_t p2 = ((w >> 8) & m) | mag, p3 = ((w >> 12) & m) | mag;  // (v2, v6), (v3, v7)
  const uint32_t q[4] = {__byte_perm(p0, p1, 0x5410), __byte_perm(p2, p3, 0x5410), __byte_perm(p0, p1, 0x7632),
                         __byte_perm(p2, p3, 0x7632)};
  const __nv_bfloat162 k128 = as_bf2(mag);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = as_u32(__hfma2(__hsub2(as_bf2(q[i]), k128), s2, b2));
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Eight 8-bit values of two words -> four bf16x2 words s * q + b.  A byte
// permute places each value in the mantissa of 2^23; s * q is exact in
// float32, so the FMA rounds once before the pairwise bf16 rounding.
__device__ __forceinline__ uint4 dequant_words8(uint32_t w0, uint32_t w1, float s, float b) {
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w = i < 2 ? w0 : w1;
    const int j = 2 * (i & 1);
    const float q0 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540 + j)) - 8388608.f;
    const float q1 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7541 + j)) - 8388608.f;
    o[i] = cvt_bf16x2(fmaf(s, q0, b), fmaf(s, q1, b));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void __launch_bounds__(kQThreads, 1) qlinear_kernel(const __grid_constant__ CUtensorMap amap,
                                                               const __grid_constant__ CUtensorMap wmap,
                                                               const __grid_constant__ CUtensorMap omap,
                                                               const __grid_constant__ CUtensorMap smap,
                                                               const __grid_constant__ CUtensorMap bmap,
                                                               const QParams p) {
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
    // The dequantizing warps arrive one by one (no CTA-wide barrier per K-block).
    for (int i = 0; i < Q_NBARS; ++i) {
      uint32_t count = 1;
      if (i >= Q_EMPTY0 && i < Q_EMPTY0 + kAStages) count = 1 + kDqWarps;  // MMA commit + every dequantizing warp
      if ((i >= Q_BFULL0 && i < Q_BFULL0 + kBStages) || i >= Q_SCEMPTY0) count = kDqWarps;
      mbar_init(&bars[i], count);
    }
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&amap);
      prefetch_tensormap(&wmap);
      if (p.scale_tma) {
        prefetch_tensormap(&smap);
        if (p.biases) prefetch_tensormap(&bmap);
      }
      int issued = 0, sc_issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kAStages;
        if (p.scale_tma && (kb & ((1 << p.sshift) - 1)) == 0) {
          // the next tile of scales and biases (8 groups), double-buffered
          const int tile = kb >> p.sshift, st = tile & 1;
          if (tile >= 2 && !mbar_wait(&bars[Q_SCEMPTY0 + st], (uint32_t)((tile / 2 - 1) & 1), kQWaitNs))
            q_record(&abort_flag);
          if (abort_flag) break;
          mbar_arrive_expect_tx(&bars[Q_SCFULL0 + st], p.biases ? 2 * kScTile : kScTile);
          tma_load_2d(base + QOFF_SC + st * 2 * kScTile, &smap, &bars[Q_SCFULL0 + st], tile * 8, (int)n0);
          if (p.biases)
            tma_load_2d(base + QOFF_SC + st * 2 * kScTile + kScTile, &bmap, &bars[Q_SCFULL0 + st], tile * 8, (int)n0);
          ++sc_issued;
        }
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
      if (abort_flag) {
        for (int kb = issued - kAStages < 0 ? 0 : issued - kAStages; kb < issued; ++kb)
          mbar_wait(&bars[Q_FULL0 + kb % kAStages], (uint32_t)((kb / kAStages) & 1), kQWaitNs);
        for (int tile = sc_issued - 2 < 0 ? 0 : sc_issued - 2; tile < sc_issued; ++tile)
          mbar_wait(&bars[Q_SCFULL0 + (tile & 1)], (uint32_t)((tile / 2) & 1), kQWaitNs);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, QBN);
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
        for (int ks = 0; ks < QBK / 16; ++ks) {
          const uint64_t bd = sdesc_sw128(b + ks * 32);
          mma_bf16(tmem, sdesc_sw128(a + ks * 32), bd, idesc, kb > 0 || ks > 0);                   // rows 0-127
          mma_bf16(tmem + QBN, sdesc_sw128(a + 128 * 128 + ks * 32), bd, idesc, kb > 0 || ks > 0);  // rows 128-255
        }
        mma_commit(&bars[Q_EMPTY0 + s]);
        mma_commit(&bars[Q_BEMPTY0 + sb]);
      }
      // The accumulators are complete (or, after an abort, every MMA issued
      // has finished) when this commit's barrier completes.
      mma_commit(&bars[Q_ACC]);
      if (kb < nk) mbar_wait(&bars[Q_ACC], 0, kQWaitNs);
    }
  } else {
    // ------------------------------------------- dequantization, then epilogue
    const int t = tid - 64;
    const int r = t & (QBN - 1), h = t >> 8;  // weight row of the tile, 32-value half of each K-block
    const int64_t row = n0 + r;
    const bool live = row < p.n;
    const int groups = (int)(p.k >> p.gshift);
    const __nv_bfloat16* srow = p.scales + (live ? row : 0) * groups;
    const __nv_bfloat16* brow = p.biases ? p.biases + (live ? row : 0) * groups : nullptr;
    // (scale, bias) of this thread's half of K-block kb; rows past n get
    // zeros, so their (zero-filled) weights dequantize to 0.
    auto load_sb = [&](int kb, __nv_bfloat16& sv, __nv_bfloat16& bv) {
      const int g = (kb * QBK + h * 32) >> p.gshift;
      sv = live ? srow[g] : __float2bfloat16_rn(0.f);
      bv = (live && brow) ? brow[g] : __float2bfloat16_rn(0.f);
    };
    // Byte offsets of this thread's four 16-byte chunks (values 32h + 8j ..)
    // in a 128-byte-swizzled K-major B tile.
    uint32_t boff[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) boff[j] = sw128_chunk(QBN, r, 0, 4 * h + j);
    // Scales and biases ride kScaleAhead K-blocks ahead in a register ring
    // (the loop is unrolled by the ring's depth, so no slot is copied while
    // its load is in flight): one block ahead, each block waited for a
    // global-memory round trip.
    __nv_bfloat16 sr[kScaleAhead], br[kScaleAhead];
#pragma unroll
    for (int j = 0; j < kScaleAhead; ++j)
      if (j < nk && !p.scale_tma) load_sb(j, sr[j], br[j]);
    bool ok = true, stop = false;
    for (int kbase = 0; kbase < nk && !stop; kbase += kScaleAhead)
#pragma unroll
    for (int j = 0; j < kScaleAhead; ++j) {
      const int kb = kbase + j;
      if (kb >= nk) break;
      const int s = kb % kAStages, sb = kb % kBStages;
      __nv_bfloat16 s_cur, b_cur;
      const int tile = kb >> p.sshift;
      const int in_tile = kb & ((1 << p.sshift) - 1);
      if (p.scale_tma) {
        // this row's group within the tile: rows past n were zero-filled
        const unsigned char* sc = base + QOFF_SC + (tile & 1) * 2 * kScTile + r * 16 +
                                  2 * (((kb * QBK + h * 32) >> p.gshift) - 8 * tile);
        ok = in_tile != 0 || mbar_wait(&bars[Q_SCFULL0 + (tile & 1)], (uint32_t)((tile >> 1) & 1), kQWaitNs);
        s_cur = *reinterpret_cast<const __nv_bfloat16*>(sc);
        b_cur = p.biases ? *reinterpret_cast<const __nv_bfloat16*>(sc + kScTile) : __float2bfloat16_rn(0.f);
      } else {
        ok = true;
        s_cur = sr[j];
        b_cur = br[j];
        if (kb + kScaleAhead < nk) load_sb(kb + kScaleAhead, sr[j], br[j]);
      }
      ok = ok && mbar_wait(&bars[Q_FULL0 + s], (uint32_t)((kb / kAStages) & 1), kQWaitNs) &&
           (kb < kBStages || mbar_wait(&bars[Q_BEMPTY0 + sb], (uint32_t)((kb / kBStages - 1) & 1), kQWaitNs));
      if (!ok) q_record(&abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {  // the warp's lanes leave together
        stop = true;
        break;
      }
      const unsigned char* wsrc = base + QOFF_W + s * kWTile + (size_t)r * wbytes + h * (wbytes / 2);
      unsigned char* bdst = base + QOFF_B + sb * kBTile;
      if (p.bits == 4) {
        const uint4 w = *reinterpret_cast<const uint4*>(wsrc);
        const __nv_bfloat162 s2 = __bfloat162bfloat162(s_cur), b2 = __bfloat162bfloat162(b_cur);
        const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(bdst + boff[j]) = dequant_word4(wd[j], s2, b2);
      } else {
        const uint4 w01 = reinterpret_cast<const uint4*>(wsrc)[0], w23 = reinterpret_cast<const uint4*>(wsrc)[1];
        const float sv = __bfloat162float(s_cur), bv = __bfloat162float(b_cur);
        *reinterpret_cast<uint4*>(bdst + boff[0]) = dequant_words8(w01.x, w01.y, sv, bv);
        *reinterpret_cast<uint4*>(bdst + boff[1]) = dequant_words8(w01.z, w01.w, sv, bv);
        *reinterpret_cast<uint4*>(bdst + boff[2]) = dequant_words8(w23.x, w23.y, sv, bv);
        *reinterpret_cast<uint4*>(bdst + boff[3]) = dequant_words8(w23.z, w23.w, sv, bv);
      }
      // each lane's writes reach the async proxy; the warp's lane 0 arrives for it
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bars[Q_BFULL0 + sb]);  // this warp's rows of the operand are ready
        mbar_arrive(&bars[Q_EMPTY0 + s]);   // and its packed weights are read
        if (p.scale_tma && (in_tile == (1 << p.sshift) - 1 || kb == nk - 1))
          mbar_arrive(&bars[Q_SCEMPTY0 + (tile & 1)]);  // and the tile's scales
      }
    }

    // ------------------------------------------------------------ epilogue
    // Warp w reads TMEM lanes 32 (w % 4) .. and columns 128 cb .. 128 cb + 127
    // (cb = (w - 2) / 4): accumulator cb / 2 (tile rows 128 (cb / 2) ..),
    // output columns 128 (cb % 2) ..; the staging (over the A and W rings,
    // idle once the accumulators are complete) holds eight 128 x 64
    // sub-tiles, accumulator-major.
    ok = !abort_flag && mbar_wait(&bars[Q_ACC], 0, kQWaitNs);
    if (!ok) q_record(&abort_flag);
    if (!named_sync_or(1, kDqThreads, !ok)) {
      tc_fence_after();
      const int q = warp & 3, cb = (warp - 2) >> 2;
      const int orow = q * 32 + lane;
      const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + cb * 128;
#pragma unroll 1
      for (int jj = 0; jj < 2; ++jj) {
        float v[64];
        tmem_ld32(tq + jj * 64, *reinterpret_cast<float(*)[32]>(v));
        tmem_ld32(tq + jj * 64 + 32, *reinterpret_cast<float(*)[32]>(v + 32));
        tmem_wait_ld();
        unsigned char* st = base + QOFF_A + (uint32_t)(cb * 2 + jj) * kOutSub;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 o = make_uint4(cvt_bf16x2(v[8 * c], v[8 * c + 1]), cvt_bf16x2(v[8 * c + 2], v[8 * c + 3]),
                                     cvt_bf16x2(v[8 * c + 4], v[8 * c + 5]), cvt_bf16x2(v[8 * c + 6], v[8 * c + 7]));
          *reinterpret_cast<uint4*>(st + sw128_chunk(128, orow, 0, c)) = o;
        }
      }
      fence_async_smem();
      named_sync(1, kDqThreads);
      if (t == 0) {
        for (int sub = 0; sub < 8; ++sub) {
          const int64_t orow0 = m0 + 128 * (sub >> 2), ocol0 = n0 + 64 * (sub & 3);
          if (orow0 < p.m && ocol0 < p.n)
            tma_store_2d(&omap, base + QOFF_A + sub * kOutSub, (int)ocol0, (int)orow0);
        }
        bulk_commit_group();
        bulk_wait_group_read0();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------
// Decode and small batches: up to 16 tokens.  The weights stream from HBM
// once; each warp owns 16 weight rows and a strided share of K, dequantizes
// straight into the A fragments of mma.sync m16n8k16 (A = 16 weight rows x 16
// K, B = 16 K x 8 tokens; one or two token blocks) and accumulates in
// float32; the CTA's warps then add their K shares in shared memory.  The
// register-fed form needs no shared-memory round trip of the weights, which
// a tcgen05 operand would; on this part each further token block costs about
// as much as the first, so beyond two the tiled GEMM takes over.
//
// Inside each run of 8 consecutive K the fragment takes the values in the
// order (0, 4, 1, 5, 2, 6, 3, 7): one AND-OR of a 4-bit word yields exactly
// the pairs (j, j + 4).  A dot product does not depend on the order of K, so
// x is staged in shared memory in that same order and the products match.
// ---------------------------------------------------------------------------
constexpr int kGvMaxTokens = 16;  // beyond two token blocks the tiled GEMM is faster
constexpr size_t kGvMaxSmem = 220 * 1024;  // staged x: (m + 1) x k bf16

struct GvParams {
  int64_t m, n, k;
  const __nv_bfloat16* x;
  int64_t x_stride;
  const uint32_t* w;
  const __nv_bfloat16* scales;
  const __nv_bfloat16* biases;
  __nv_bfloat16* out;
  int64_t out_stride;
  int gshift, row_groups;  // row_groups of 16 rows per CTA; the warps split K (warps / row_groups) ways
};

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Values (j, j + 4) of a 4-bit word, j = 0..3, as bf16x2 s * q + b.
__device__ __forceinline__ void gv_pairs4(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 b2, uint32_t (&o)[4]) {
  const uint32_t m = 0x000F000Fu, mag = 0x43004300u;
  const __nv_bfloat162 k128 = as_bf2(mag);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    o[j] = as_u32(__hfma2(__hsub2(as_bf2(((w >> (4 * j)) & m) | mag), k128), s2, b2));
}

// Values (j, j + 4) of the 8-bit words w0 (values 0-3) and w1 (4-7).
__device__ __forceinline__ void gv_pairs8(uint32_t w0, uint32_t w1, float s, float b, uint32_t (&o)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float q0 = __uint_as_float(__byte_perm(w0, 0x4B000000u, 0x7540 + j)) - 8388608.f;
    const float q1 = __uint_as_float(__byte_perm(w1, 0x4B000000u, 0x7540 + j)) - 8388608.f;
    o[j] = cvt_bf16x2(fmaf(s, q0, b), fmaf(s, q1, b));
  }
}

template <int BITS, int WARPS, int NT>
__global__ void __launch_bounds__(WARPS * 32, WARPS == 8 ? (NT == 1 ? 3 : 2) : 1) qgemv_kernel(const GvParams p) {
  griddep_wait();  // launched as a dependent of the kernel before it
  griddep_launch_dependents();
  // [m + 1][k / 8] runs of 8, each in the order (0, 4, 1, 5, 2, 6, 3, 7); row m is zeros.
  // After the main loop the same memory holds the warps' partial sums.
  extern __shared__ uint4 xs[];
  float(*red)[NT * 4][32] = reinterpret_cast<float(*)[NT * 4][32]>(xs);
  constexpr int U = BITS == 4 ? 4 : 2;  // chunks whose loads are in flight together
  constexpr int NW = BITS / 4;          // uint4 per row and chunk: the thread's 32 values
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int m = (int)p.m, k = (int)p.k, runs = k / 8;

  const int ksplit = WARPS / p.row_groups;
  const int rg = warp / ksplit, ks = warp % ksplit;
  const int64_t rowA = ((int64_t)blockIdx.x * p.row_groups + rg) * 16 + g, rowB = rowA + 8;
  const bool liveA = rowA < p.n, liveB = rowB < p.n;
  const int groups = k >> p.gshift;
  // Rows past n read row 0 with a zero scale and bias: their products are 0.
  const int64_t ra = liveA ? rowA : 0, rb = liveB ? rowB : 0;
  const uint4* wA = reinterpret_cast<const uint4*>(p.w) + ra * (k * BITS / 128);
  const uint4* wB = reinterpret_cast<const uint4*>(p.w) + rb * (k * BITS / 128);
  const __nv_bfloat16* sA = p.scales + ra * groups;
  const __nv_bfloat16* sB = p.scales + rb * groups;
  const __nv_bfloat16* bA = p.biases ? p.biases + ra * groups : nullptr;
  const __nv_bfloat16* bB = p.biases ? p.biases + rb * groups : nullptr;
  const __nv_bfloat16 zero = __float2bfloat16_rn(0.f);
  const int nchunks = (k + 127) / 128;  // 128 K per warp step: 32 per thread

  uint4 va[U][NW], vb[U][NW];
  __nv_bfloat16 sa[U], sb[U], ba[U], bb[U];
  bool on[U];  // this lane's 32 values exist (lanes t4 >= 2 of a ragged last chunk, k % 128 == 64, have none)
  auto load_batch = [&](int c0) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u * ksplit;
      if (c >= nchunks) continue;  // uniform across the warp
      const int kk = c * 128 + 32 * t4;
      on[u] = kk < k;
      const int off = on[u] ? kk * BITS / 128 : 0;  // uint4 offset of the lane's 32 values in the row
      const int grp = on[u] ? kk >> p.gshift : 0;
#pragma unroll
      for (int e = 0; e < NW; ++e) {
        va[u][e] = wA[off + e];
        vb[u][e] = wB[off + e];
      }
      sa[u] = (on[u] && liveA) ? sA[grp] : zero;
      sb[u] = (on[u] && liveB) ? sB[grp] : zero;
      ba[u] = (on[u] && liveA && bA) ? bA[grp] : zero;
      bb[u] = (on[u] && liveB && bB) ? bB[grp] : zero;
    }
  };

  // The first batch of weights does not need x: its loads go out before x
  // is staged.
  int c0 = ks;
  load_batch(c0);
  for (int tok = 0; tok < m; ++tok)
    for (int r = tid; r < runs; r += WARPS * 32) {
      const uint4 v = *reinterpret_cast<const uint4*>(p.x + tok * p.x_stride + 8 * r);
      xs[tok * runs + r] = make_uint4(__byte_perm(v.x, v.z, 0x5410), __byte_perm(v.x, v.z, 0x7632),
                                      __byte_perm(v.y, v.w, 0x5410), __byte_perm(v.y, v.w, 0x7632));
    }
  for (int r = tid; r < runs; r += WARPS * 32) xs[m * runs + r] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  // token block t: tokens 8 t + g; tokens past m read the zero row
  const uint4* xrow[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) xrow[t] = xs + (8 * t + g < m ? 8 * t + g : m) * runs + t4 * 4;
  const uint4* xzero = xs + m * runs;

  float acc[NT][4] = {};
  for (; c0 < nchunks; c0 += ksplit * U) {
    if (c0 != ks) load_batch(c0);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      // mma.sync is warp-wide: skip only whole chunks past the end (uniform
      // across the warp); lanes without values have zero scales and biases
      // and read the zero x row.
      const int c = c0 + u * ksplit;
      if (c >= nchunks) continue;
      const int xoff = on[u] ? c * 16 : 0;
      if (BITS == 4) {
        const __nv_bfloat162 sa2 = __bfloat162bfloat162(sa[u]), ba2 = __bfloat162bfloat162(ba[u]);
        const __nv_bfloat162 sb2 = __bfloat162bfloat162(sb[u]), bb2 = __bfloat162bfloat162(bb[u]);
        const uint32_t wa[4] = {va[u][0].x, va[u][0].y, va[u][0].z, va[u][0].w};
        const uint32_t wb[4] = {vb[u][0].x, vb[u][0].y, vb[u][0].z, vb[u][0].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t pa[4], pb[4];
          gv_pairs4(wa[j], sa2, ba2, pa);
          gv_pairs4(wb[j], sb2, bb2, pb);
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const uint4 xv = on[u] ? xrow[t][xoff + j] : xzero[j];
            mma_16816(acc[t], pa[0], pb[0], pa[1], pb[1], xv.x, xv.y);
            mma_16816(acc[t], pa[2], pb[2], pa[3], pb[3], xv.z, xv.w);
          }
        }
      } else {
        const float fsa = __bfloat162float(sa[u]), fba = __bfloat162float(ba[u]);
        const float fsb = __bfloat162float(sb[u]), fbb = __bfloat162float(bb[u]);
        const uint32_t wa[8] = {va[u][0].x, va[u][0].y, va[u][0].z, va[u][0].w,
                                va[u][NW - 1].x, va[u][NW - 1].y, va[u][NW - 1].z, va[u][NW - 1].w};
        const uint32_t wb[8] = {vb[u][0].x, vb[u][0].y, vb[u][0].z, vb[u][0].w,
                                vb[u][NW - 1].x, vb[u][NW - 1].y, vb[u][NW - 1].z, vb[u][NW - 1].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t pa[4], pb[4];
          gv_pairs8(wa[2 * j], wa[2 * j + 1], fsa, fba, pa);
          gv_pairs8(wb[2 * j], wb[2 * j + 1], fsb, fbb, pb);
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const uint4 xv = on[u] ? xrow[t][xoff + j] : xzero[j];
            mma_16816(acc[t], pa[0], pb[0], pa[1], pb[1], xv.x, xv.y);
            mma_16816(acc[t], pa[2], pb[2], pa[3], pb[3], xv.z, xv.w);
          }
        }
      }
    }
  }

  __syncthreads();  // x is dead: its memory takes the partial sums
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) red[warp][4 * t + i][lane] = acc[t][i];
  __syncthreads();
  if (ks == 0) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      float sum[4] = {0.f, 0.f, 0.f, 0.f};
      for (int w = warp; w < warp + ksplit; ++w)
#pragma unroll
        for (int i = 0; i < 4; ++i) sum[i] += red[w][4 * t + i][lane];
      // sum[0], sum[1]: row g, tokens 8 t + 2 t4, + 1; sum[2], sum[3]: row g + 8
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tok = 8 * t + 2 * t4 + (i & 1);
        const int64_t row = i < 2 ? rowA : rowB;
        if (tok < m && row < p.n) p.out[tok * p.out_stride + row] = __float2bfloat16_rn(sum[i]);
      }
    }
  }
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
  p->gshift = a->group_size == 32 ? 5 : a->group_size == 64 ? 6 : 7;
  p->sshift = p->gshift - 3;
  // scale tiles by TMA when a row of scales is a whole number of 16-byte units
  p->scale_tma = (a->k / a->group_size) % 8 == 0 && a16(a->scales) && (!a->biases || a16(a->biases));
  return GDN_OK;
}

gdn_status q_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return GDN_OK;
  return set_error(GDN_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace

template <int BITS, int WARPS, int NT>
gdn_status gv_launch_one(const GvParams& g, unsigned grid, size_t smem, cudaStream_t cs) {
  static DeviceFlags attr;
  const gdn_status st =
      q_cuda(ensure_smem_attr(qgemv_kernel<BITS, WARPS, NT>, kGvMaxSmem, attr), "quantized_linear attribute");
  if (st != GDN_OK) return st;
  return q_cuda(launch_dependent(qgemv_kernel<BITS, WARPS, NT>, dim3(grid), dim3(WARPS * 32), smem, cs, g),
                "quantized_linear launch");
}

template <int BITS, int WARPS>
gdn_status gv_launch(int nt, const GvParams& g, unsigned grid, size_t smem, cudaStream_t cs) {
  if (nt == 1) return gv_launch_one<BITS, WARPS, 1>(g, grid, smem, cs);
  return gv_launch_one<BITS, WARPS, 2>(g, grid, smem, cs);
}

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
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  const size_t gv_x = (size_t)(a->m + 1) * (size_t)a->k * 2;
  if (a->m <= gdn::kGvMaxTokens && gv_x <= gdn::kGvMaxSmem) {
    // up to 16 tokens: the weights stream once through the register-fed GEMV
    gdn::GvParams g;
    g.m = a->m;
    g.n = a->n;
    g.k = a->k;
    g.x = static_cast<const __nv_bfloat16*>(a->x);
    g.x_stride = a->x_stride_m;
    g.w = a->w;
    g.scales = p.scales;
    g.biases = p.biases;
    g.out = static_cast<__nv_bfloat16*>(a->out);
    g.out_stride = a->out_stride_m;
    g.gshift = p.gshift;
    const int64_t rows16 = (a->n + 15) / 16;
    int warps = 8;
    g.row_groups = 1;
    if (rows16 >= 4 * 148) g.row_groups = 2;
    else if (a->k >= 16 * 128) warps = 16;
    const int nt = a->m <= 8 ? 1 : 2;
    const unsigned grid = (unsigned)((rows16 + g.row_groups - 1) / g.row_groups);
    const size_t red = (size_t)warps * nt * 4 * 32 * sizeof(float);
    const size_t smem = gv_x > red ? gv_x : red;
    if (a->bits == 4)
      return warps == 8 ? gdn::gv_launch<4, 8>(nt, g, grid, smem, cs) : gdn::gv_launch<4, 16>(nt, g, grid, smem, cs);
    return warps == 8 ? gdn::gv_launch<8, 8>(nt, g, grid, smem, cs) : gdn::gv_launch<8, 16>(nt, g, grid, smem, cs);
  }
  CUtensorMap amap, wmap, omap;
  const int64_t kw = a->k * a->bits / 32;  // words per weight row
  if (!gdn::q_map(&amap, a->x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a->k, a->m, a->x_stride_m * 2, 64, gdn::QBM, true) ||
      !gdn::q_map(&wmap, a->w, CU_TENSOR_MAP_DATA_TYPE_UINT32, kw, a->n, kw * 4, 64 * a->bits / 32, 256, false) ||
      !gdn::q_map(&omap, a->out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, a->n, a->m, a->out_stride_m * 2, 64, 128, true))
    return gdn::set_error(GDN_ECUDA, "quantized_linear: tensor map encoding failed");
  static gdn::DeviceFlags attr;
  st = gdn::q_cuda(gdn::ensure_smem_attr(gdn::qlinear_kernel, gdn::kQSmem, attr), "quantized_linear attribute");
  if (st != GDN_OK) return st;
  CUtensorMap smap, bmap;
  std::memset(&smap, 0, sizeof(smap));
  std::memset(&bmap, 0, sizeof(bmap));
  const int64_t groups = a->k / a->group_size;
  if (p.scale_tma &&
      (!gdn::q_map(&smap, a->scales, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, groups, a->n, groups * 2, 8, gdn::QBN, false) ||
       (a->biases &&
        !gdn::q_map(&bmap, a->biases, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, groups, a->n, groups * 2, 8, gdn::QBN, false))))
    return gdn::set_error(GDN_ECUDA, "quantized_linear: tensor map encoding failed");
  const dim3 grid((unsigned)((a->n + gdn::QBN - 1) / gdn::QBN), (unsigned)((a->m + gdn::QBM - 1) / gdn::QBM));
  if (grid.y > 65535) return gdn::set_error(GDN_EUNSUPPORTED, "m too large for one call (%lld)", (long long)a->m);
  gdn::qlinear_kernel<<<grid, gdn::kQThreads, gdn::kQSmem, cs>>>(amap, wmap, omap, smap, bmap, p);
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
