/*
 * gdn_api.h -- C ABI of the B200 gated-delta (GatedDeltaNet) library,
 * libgdn_b200.so.
 *
 * The reference (conferencebeefwood46/mlx-lean-moe) reaches this operator
 * through one Python function and its accelerator hook:
 *
 *   gated_delta_scan(q, k, v, g, beta, state, *, use_kernel=True)
 *       -> (y, new_state)        src/mlx_lean_moe/model/qwen3_5/gated_delta.py:44-90
 *   gated_delta_scan_metal(q, k, v, g, beta, state)
 *       -> (y, new_state)        src/mlx_lean_moe/model/qwen3_5/_gated_delta_metal.py:95-114
 *
 * gdn_scan / gdn_decode below replace that hook (gated_delta.py:88): the
 * reference's Python checks shapes, then hands row-contiguous arrays to a
 * device kernel that returns y and a new state.  gdn_fused_block replaces the
 * body of Qwen3_5LinearAttention.__call__ between the input projections and
 * out_proj (linear_attention.py:103-124), and gdn_forget_gate replaces
 * forget_gate (gated_delta.py:14-21).
 *
 * Conventions
 *  - Every tensor pointer is a DEVICE pointer; strides are in ELEMENTS; the
 *    innermost (feature) dimension is always contiguous (the reference's
 *    kernel copies strided inputs to row-contiguous ones,
 *    _gated_delta_metal.py:43 "ensure_row_contiguous=True").
 *  - Work is enqueued on the caller's stream; nothing is synchronised and
 *    nothing is allocated: scratch memory comes from the caller
 *    (gdn_*_workspace_size).  Calls on one stream run in order.
 *  - Every function returns a gdn_status; on failure
 *    gdn_last_error() (thread-local) says why.  Shape/dtype errors are found
 *    on the host before anything is launched, like the reference's
 *    ValueErrors (gated_delta.py:57-79).  Nothing aborts the process.
 *  - State layout is the reference's RecurrentCache (recurrent_cache.py:27-32):
 *    ssm state [Hv, Dv, Dk] float32 per sequence, Dk contiguous; batches stack
 *    a leading sequence axis [B, Hv, Dv, Dk].  conv state [K-1, C] per
 *    sequence, C = 2*Hk*Dk + Hv*Dv in the channel order q | k | v.
 *  - GQA: value head h reads key head h / (Hv / Hk) (repeat-interleave,
 *    gated_delta.py:97-101).
 */
#ifndef GDN_API_H
#define GDN_API_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_API_VERSION 1

typedef enum {
  GDN_OK = 0,
  GDN_EINVAL = 1,       /* bad shape, stride, pointer or size            */
  GDN_EUNSUPPORTED = 2, /* valid, but no kernel for this dtype/shape     */
  GDN_ECUDA = 3,        /* a CUDA runtime call or launch failed          */
  GDN_ETIMEOUT = 4      /* a bounded device-side wait gave up            */
} gdn_status;

typedef enum { GDN_F32 = 0, GDN_BF16 = 1, GDN_F16 = 2 } gdn_dtype;

/* The reference's g is the multiplicative decay in (0, 1]
 * (gated_delta.py:14-21, :35); the chunked form needs its log. */
typedef enum { GDN_GATE_MULT = 0, GDN_GATE_LOG = 1 } gdn_gate_kind;

typedef enum {
  GDN_ALGO_AUTO = 0,    /* library picks                                   */
  GDN_ALGO_SERIAL = 1,  /* token-serial recurrence, state in registers     */
  GDN_ALGO_CHUNKED = 2  /* chunk-64 WY/UT form on the tensor cores         */
} gdn_algo;

typedef void *gdn_stream_t; /* a cudaStream_t; NULL = legacy default stream */

/* Packed sequences.  Sequence b owns tokens [cu_seqlens[b], cu_seqlens[b+1]);
 * cu_seqlens == NULL means n_seqs sequences of n_tokens / n_seqs tokens each.
 * A sequence of length 0 copies its state through. */
typedef struct {
  int64_t n_tokens;          /* N                                            */
  int64_t n_seqs;            /* B                                            */
  const int64_t *cu_seqlens; /* device, [B + 1], or NULL                     */
  int32_t hk, hv, dk, dv;    /* key heads, value heads, key dim, value dim   */

  const void *q;             /* [N, Hk, Dk], qkv_dtype                       */
  int64_t q_stride_t, q_stride_h;
  const void *k;             /* [N, Hk, Dk], qkv_dtype                       */
  int64_t k_stride_t, k_stride_h;
  const void *v;             /* [N, Hv, Dv], qkv_dtype                       */
  int64_t v_stride_t, v_stride_h;
  const void *g;             /* [N, Hv], gate_dtype, kind = gate_kind        */
  int64_t g_stride_t;
  const void *beta;          /* [N, Hv], gate_dtype                          */
  int64_t beta_stride_t;

  const float *state_in;     /* [B, Hv, Dv, Dk] or NULL (zeros)             */
  float *state_out;          /* [B, Hv, Dv, Dk]; may equal state_in          */
  void *out;                 /* [N, Hv, Dv] contiguous, out_dtype            */

  gdn_dtype qkv_dtype;       /* F32 or BF16 (F16 accepted by the serial path)*/
  gdn_dtype gate_dtype;      /* F32 or BF16                                  */
  gdn_dtype out_dtype;       /* F32 or BF16                                  */
  gdn_gate_kind gate_kind;
  gdn_algo algo;

  void *workspace;           /* device scratch, >= gdn_scan_workspace_size   */
  size_t workspace_bytes;
} gdn_scan_args;

/* One token for each of B sequences: n_tokens == n_seqs, cu_seqlens NULL.
 * state_slots (device int32 [B], or NULL) maps sequence b to state row
 * state_slots[b] of a state pool of n_slots entries (serving caches keep one
 * pool and pass the slots of the sequences in this batch); state_in and
 * state_out then point at the pool. */
typedef struct {
  gdn_scan_args base;
  const int32_t *state_slots;
  int64_t n_slots;
} gdn_decode_args;

/* The linear-attention layer from its projections to the gated norm
 * (linear_attention.py:103-124): causal depthwise conv (kernel K) + SiLU over
 * [conv_state ; q|k|v], q/k rms-norm with eps 1e-6 and scales Dk^-1, Dk^-1/2,
 * g = -exp(A_log) softplus(a + dt_bias) (log form), beta = sigmoid(b), the
 * gated-delta scan, and out = silu(z) * rms_norm(y, norm_w, eps). */
typedef struct {
  int64_t n_tokens, n_seqs;
  const int64_t *cu_seqlens;   /* as in gdn_scan_args                       */
  int32_t hk, hv, dk, dv, conv_kernel;

  const void *mixed;           /* [N, W]: q | k | v | z | b | a, widths
                                  Hk*Dk, Hk*Dk, Hv*Dv, Hv*Dv, Hv, Hv        */
  int64_t mixed_stride_t;      /* >= W                                       */
  gdn_dtype act_dtype;         /* dtype of mixed and out: F32 or BF16       */

  const float *conv_w;         /* [C, K] float32                             */
  const void *conv_state_in;   /* [B, K-1, C] conv_state_dtype, or NULL      */
  void *conv_state_out;        /* [B, K-1, C]; may equal conv_state_in       */
  gdn_dtype conv_state_dtype;  /* F32 or BF16                                */

  const float *A_log, *dt_bias;/* [Hv] float32                               */
  const float *norm_w;         /* [Dv] float32                               */
  float eps;                   /* gated rms-norm epsilon (rms_norm_eps)      */

  const float *state_in;       /* [B, Hv, Dv, Dk] or NULL                    */
  float *state_out;            /* may equal state_in                         */
  void *out;                   /* [N, Hv, Dv] act_dtype                      */
  gdn_algo algo;

  void *workspace;
  size_t workspace_bytes;
} gdn_block_args;

/* Library version (GDN_API_VERSION). */
int gdn_version(void);

/* Reason for the last failure on this thread ("" if none). */
const char *gdn_last_error(void);

/* Bytes of scratch gdn_scan needs for these arguments (0 for the serial
 * path).  Replaces nothing in the reference (MLX allocates internally). */
gdn_status gdn_scan_workspace_size(const gdn_scan_args *args, size_t *bytes);

/* gated_delta_scan over B packed sequences: y and the final states.
 * Replaces gated_delta_scan_metal, _gated_delta_metal.py:95-114 (and the ops
 * fallback _gated_delta_scan_ops, gated_delta.py:93-109). */
gdn_status gdn_scan(const gdn_scan_args *args, gdn_stream_t stream);

/* One decode step for B sequences (the T == 1 case of gdn_scan, HBM-bound).
 * Replaces the per-token call of gated_delta_scan made during decode
 * (linear_attention.py:118-119 with seq_len == 1). */
gdn_status gdn_decode(const gdn_decode_args *args, gdn_stream_t stream);

/* forget_gate (gated_delta.py:14-21): g[n, h] = exp(-exp(A_log[h]) *
 * softplus(a[n, h] + dt_bias[h])), or its log when kind == GDN_GATE_LOG.
 * a: [n, hv] in a_dtype (row stride a_stride_t); g: [n, hv] float32. */
gdn_status gdn_forget_gate(const void *a, gdn_dtype a_dtype, int64_t a_stride_t,
                           int64_t n, int32_t hv, const float *A_log,
                           const float *dt_bias, float *g, gdn_gate_kind kind,
                           gdn_stream_t stream);

/* Bytes of scratch gdn_fused_block needs. */
gdn_status gdn_block_workspace_size(const gdn_block_args *args, size_t *bytes);

/* The fused linear-attention block (see gdn_block_args).  Replaces
 * Qwen3_5LinearAttention.__call__ from the projections to the gated norm,
 * linear_attention.py:103-124, and its RecurrentCache.update (:120). */
gdn_status gdn_fused_block(const gdn_block_args *args, gdn_stream_t stream);

/* Size of the device scratch array behind gdn_fused_block_noalloc: 16 MiB
 * (about 500 tokens of scratch at the Qwen3.5 linear-attention shape, 16/32
 * heads of 128, bf16 activations). */
#define GDN_NOALLOC_SCRATCH_BYTES (16u << 20)

/* gdn_fused_block for callers that cannot allocate device memory.  It has no
 * counterpart in the reference (MLX allocates internally).
 *
 * Some callers cannot hand the library a workspace: a host bound to this
 * library through a plain C FFI (Go, Java, Rust, a game or embedded engine)
 * has no device allocator of its own and would need a cudaMalloc/cudaFree
 * per call, which synchronises the whole device and stalls every stream in a
 * serving loop; a server that reserves its entire device budget at start-up
 * (weights, state pools) has no headroom for a per-call allocation at all.
 * This entry point takes the same arguments as gdn_fused_block, ignores
 * args->workspace / workspace_bytes, and instead uses one scratch array of
 * GDN_NOALLOC_SCRATCH_BYTES compiled into the library as a __device__
 * variable.  Every GPU on which the library is loaded holds that array until
 * the process exits.  The call allocates nothing: no cudaMalloc, no cudaFree,
 * no allocating library routine.
 *
 *  - Calls whose scratch need (gdn_block_workspace_size) exceeds
 *    GDN_NOALLOC_SCRATCH_BYTES are rejected with GDN_EUNSUPPORTED before
 *    anything runs; split them into calls over fewer tokens.
 *  - The first call on each device looks up the array's device address
 *    (cudaGetSymbolAddress, with that device current) and caches it; make
 *    that first call before any stream capture.  The cache is keyed by the
 *    device ordinal and is never refreshed: after cudaDeviceReset (or
 *    anything else that destroys and recreates the device's primary
 *    context) the cached address is stale, so a process that resets a
 *    device must not call this entry point on it again.
 *  - All calls share the one array.  Calls that can overlap on the GPU
 *    (different streams, or several host threads) race on it: serialise them,
 *    e.g. on one stream.  The array keeps the last call's data; nothing in it
 *    needs to start at zero, since every scratch value is written before it
 *    is read within a call. */
gdn_status gdn_fused_block_noalloc(const gdn_block_args *args, gdn_stream_t stream);

/* A linear projection with affine-quantized weights (the layer's in_proj_* /
 * out_proj): out[m, n] = sum_k x[m, k] * W[n, k] with
 * W[n, k] = scales[n, k / group_size] * q[n, k] + biases[n, k / group_size]
 * (biases optional: 0), the unsigned `bits`-bit values q packed into uint32
 * words along k, value j of a word in bits [j * bits, (j + 1) * bits).
 *   x:      [m, k], row stride x_stride_m (elements, multiple of 8), bf16
 *   w:      [n, k * bits / 32] uint32, rows contiguous
 *   scales: [n, k / group_size], biases the same (or NULL), bf16
 *   out:    [m, n], row stride out_stride_m (elements, multiple of 8), bf16
 * bits 4 or 8; group_size 32, 64 or 128; k a multiple of 64 and of
 * group_size; x, w and out 16-byte aligned.  Accumulation in float32; each
 * dequantized weight is rounded to bf16 before the product.  Up to 16 rows of
 * x (decode) stream the weights once through a register-fed kernel; more
 * rows run the tiled tensor-core GEMM.  Replaces quantized_linear /
 * mx.quantized_matmul (model/moe_block.py:23-50) for the affine mode. */
typedef struct {
  int64_t m, n, k;
  const void *x;
  int64_t x_stride_m;
  const uint32_t *w;
  const void *scales;
  const void *biases;
  int32_t bits, group_size;
  void *out;
  int64_t out_stride_m;
} gdn_qlinear_args;

gdn_status gdn_quantized_linear(const gdn_qlinear_args *args, gdn_stream_t stream);

/* W (as above) dequantized into a dense [n, k] matrix of out_dtype (float32
 * or bf16) with row stride k: the same weights as gdn_quantized_linear uses,
 * for callers whose activations are not bf16. */
gdn_status gdn_dequantize(const gdn_qlinear_args *args, gdn_dtype out_dtype, void *dense,
                          gdn_stream_t stream);

/* The softmax-attention layer between its projections (the reference's
 * Qwen3_5Attention.__call__, qw/attention.py:56-96, with GrowingKVCache,
 * cache/kv_cache.py:28-102), for one sequence:
 *   q, gate = qg split per head; q = rope(rms_norm(q, q_norm, eps));
 *   k = rope(rms_norm(k_new, k_norm, eps)); the cache rows
 *   [cache_len - n_tokens, cache_len) receive k and v_new; then
 *   out = sdpa(q, keys, values, scale, causal) * sigmoid(gate),
 * with grouped-query heads (query head h reads key/value head
 * h / (heads / kv_heads)), the causal mask aligned to the newest query, and
 * rope rotating features [0, rotary_dim) pairwise (i, i + rotary_dim / 2) by
 * position * rope_base^(-2i / rotary_dim).  Activations and caches share
 * act_dtype (F32 or BF16); the norms and the softmax run in float32.
 *   qg:     [n_tokens, heads * 2 * head_dim]  (per head: queries | gate)
 *   k_new, v_new: [n_tokens, kv_heads * head_dim]
 *   q_norm, k_norm: [head_dim] float32
 *   k_cache, v_cache: [kv_heads, capacity, head_dim], 16-byte aligned
 *   out:    [n_tokens, heads * head_dim]
 * head_dim 32, 64, 128 or 256.  The workspace holds the rotated queries and,
 * for calls with few rows (decode), the partial rows of the key splits. */
typedef struct {
  int64_t n_tokens;          /* new tokens of this call                    */
  int64_t cache_len;         /* cached positions after this call           */
  int64_t capacity;          /* rows allocated per head in the caches      */
  int32_t heads, kv_heads, head_dim, rotary_dim;
  float rope_base, eps, scale;
  const void *qg;
  int64_t qg_stride_t;
  const void *k_new;
  int64_t k_stride_t;
  const void *v_new;
  int64_t v_stride_t;
  const float *q_norm;
  const float *k_norm;
  void *k_cache;
  void *v_cache;
  gdn_dtype act_dtype;
  void *out;
  int64_t out_stride_t;
  void *workspace;
  size_t workspace_bytes;
} gdn_attn_args;

gdn_status gdn_attention_workspace_size(const gdn_attn_args *args, size_t *bytes);
gdn_status gdn_attention(const gdn_attn_args *args, gdn_stream_t stream);

/* Head-sharded prefill with the output all-gather fused into the scan.
 *
 * The reference has no multi-device path; this is the optional all-gather of
 * head-sharded outputs (one process per GPU, each scanning whole GQA groups,
 * value heads [head0, head0 + hv) of hv_total) done by the scan kernel itself:
 * its output stage writes each finished 64-token tile of y into this rank's
 * gathered output (args->out, [N, hv_total, Dv] contiguous, out_dtype) and,
 * with 16-byte stores over NVLink, into every other rank's (peer_out: their
 * gathered outputs as mapped on this device, e.g. by gdn_ipc_import), so the
 * transfer overlaps the scan instead of following it.  Everything else is
 * gdn_scan's (the workspace is gdn_scan_workspace_size of the same args);
 * the chunked path only (bf16 q/k/v, dk == dv == 128).  A rank's buffer is
 * complete once every rank's call has completed: order its readers after a
 * cross-rank barrier (e.g. a one-element NCCL all-reduce on the stream). */
#define GDN_MAX_GATHER_PEERS 7
typedef struct {
  int32_t hv_total;            /* value heads of the gathered output          */
  int32_t head0;               /* first value head of this call within it     */
  int32_t n_peers;             /* 0 .. GDN_MAX_GATHER_PEERS                   */
  int32_t reserved;            /* 0                                           */
  void *peer_out[GDN_MAX_GATHER_PEERS]; /* 16-byte aligned                    */
} gdn_gather_args;

gdn_status gdn_scan_gathered(const gdn_scan_args *args, const gdn_gather_args *gather, gdn_stream_t stream);

/* CUDA IPC for the peer outputs above (no counterpart in the reference).
 * gdn_ipc_export writes the handle of the allocation that holds `ptr` and
 * ptr's byte offset in it; gdn_ipc_import maps a handle exported by another
 * process of this node into this one (peer access enabled) and returns the
 * address of the same byte; gdn_ipc_release unmaps it. */
#define GDN_IPC_HANDLE_BYTES 64
gdn_status gdn_ipc_export(const void *ptr, unsigned char *handle, uint64_t *offset);
gdn_status gdn_ipc_import(const unsigned char *handle, uint64_t offset, void **ptr);
gdn_status gdn_ipc_release(void *ptr, uint64_t offset);

/* Synchronises `stream`, then reports and clears any error a bounded
 * device-side wait recorded since the last call (GDN_ETIMEOUT), or a CUDA
 * error (GDN_ECUDA). */
gdn_status gdn_check_device_errors(gdn_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_API_H */
