// The C ABI of libgdn_b200 (declared in include/gdn_api.h): argument
// checks on the host, then dispatch to the kernels.  Every check runs before
// any launch, the way the reference raises ValueError before dispatching to
// its kernel (src/mlx_lean_moe/model/qwen3_5/gated_delta.py:57-79).
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include <cuda.h>
#include <string>

#include "gdn_common.cuh"
#include "gdn_testing.h"

namespace {

thread_local std::string g_last_error;

gdn_status fail(gdn_status st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return st;
}

gdn_status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return GDN_OK;
  return fail(GDN_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

size_t dtype_size(gdn_dtype d) { return d == GDN_F32 ? 4 : 2; }
bool valid_dtype(int d) { return d == GDN_F32 || d == GDN_BF16 || d == GDN_F16; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Checks shared by gdn_scan / gdn_decode; fills the internal parameter block.
// check_pointers is false for the scan inside the fused block, whose
// q/k/v/g/beta/out live in a workspace that may not be given yet (size query).
gdn_status check_scan(const gdn_scan_args* a, gdn::ScanParams* p, int64_t state_rows, bool check_pointers = true) {
  if (!a) return fail(GDN_EINVAL, "args is NULL");
  if (a->hk <= 0 || a->hv <= 0 || a->dk <= 0 || a->dv <= 0)
    return fail(GDN_EINVAL, "gated_delta_scan requires nonempty sequence and head dimensions "
                            "(hk=%d hv=%d dk=%d dv=%d)", a->hk, a->hv, a->dk, a->dv);
  if (a->hv % a->hk)
    return fail(GDN_EINVAL, "v must match q's sequence length and have a multiple of its head count "
                            "(hv=%d hk=%d)", a->hv, a->hk);
  if (a->n_tokens < 0 || a->n_seqs <= 0) return fail(GDN_EINVAL, "n_tokens must be >= 0 and n_seqs > 0");
  if (!a->cu_seqlens && a->n_tokens % a->n_seqs)
    return fail(GDN_EINVAL, "without cu_seqlens, n_tokens (%lld) must be a multiple of n_seqs (%lld)",
                (long long)a->n_tokens, (long long)a->n_seqs);
  if (!valid_dtype(a->qkv_dtype)) return fail(GDN_EINVAL, "bad qkv_dtype %d", (int)a->qkv_dtype);
  if (a->gate_dtype != GDN_F32 && a->gate_dtype != GDN_BF16)
    return fail(GDN_EUNSUPPORTED, "gate_dtype must be F32 or BF16");
  if (a->out_dtype != GDN_F32 && a->out_dtype != GDN_BF16)
    return fail(GDN_EUNSUPPORTED, "out_dtype must be F32 or BF16");
  if (a->gate_kind != GDN_GATE_MULT && a->gate_kind != GDN_GATE_LOG) return fail(GDN_EINVAL, "bad gate_kind");
  if (check_pointers && a->n_tokens > 0 && (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->out))
    return fail(GDN_EINVAL, "q, k, v, g, beta and out must be non-NULL");
  if (!a->state_out) return fail(GDN_EINVAL, "state_out must be non-NULL");
  if (!aligned16(a->state_out) || (a->state_in && !aligned16(a->state_in)))
    return fail(GDN_EINVAL, "state_in/state_out must be 16-byte aligned");
  if (a->q_stride_t < 0 || a->q_stride_h < 0 || a->k_stride_t < 0 || a->k_stride_h < 0 || a->v_stride_t < 0 ||
      a->v_stride_h < 0 || a->g_stride_t < 0 || a->beta_stride_t < 0)
    return fail(GDN_EINVAL, "strides must be non-negative");
  if (a->state_in && a->state_in != a->state_out) {
    const int64_t bytes = state_rows * a->hv * (int64_t)a->dv * a->dk * 4;
    const char* i0 = reinterpret_cast<const char*>(a->state_in);
    const char* o0 = reinterpret_cast<const char*>(a->state_out);
    if (i0 < o0 + bytes && o0 < i0 + bytes)
      return fail(GDN_EINVAL, "state_out overlaps state_in without being identical to it");
  }
  p->n_tokens = a->n_tokens;
  p->n_seqs = a->n_seqs;
  p->cu_seqlens = a->cu_seqlens;
  p->hk = a->hk;
  p->hv = a->hv;
  p->dk = a->dk;
  p->dv = a->dv;
  p->q = a->q;
  p->k = a->k;
  p->v = a->v;
  p->g = a->g;
  p->beta = a->beta;
  p->q_st = a->q_stride_t;
  p->q_sh = a->q_stride_h;
  p->k_st = a->k_stride_t;
  p->k_sh = a->k_stride_h;
  p->v_st = a->v_stride_t;
  p->v_sh = a->v_stride_h;
  p->g_st = a->g_stride_t;
  p->beta_st = a->beta_stride_t;
  p->state_in = a->state_in;
  p->state_out = a->state_out;
  p->out = a->out;
  p->qkv_dtype = a->qkv_dtype;
  p->gate_dtype = a->gate_dtype;
  p->out_dtype = a->out_dtype;
  p->gate_kind = a->gate_kind;
  p->state_slots = nullptr;
  p->workspace = a->workspace;
  p->workspace_bytes = a->workspace_bytes;
  return GDN_OK;
}

// Resolves the algorithm for a checked scan.
gdn_status pick_algo(const gdn_scan_args* a, const gdn::ScanParams& p, bool* chunked) {
  const bool can_chunk = gdn::chunked_supported(p);
  const bool can_serial = gdn::serial_supported(p.dk);
  switch (a->algo) {
    case GDN_ALGO_SERIAL:
      if (!can_serial) return fail(GDN_EUNSUPPORTED, "serial scan needs dk %% 4 == 0 and dk <= 256 (dk=%d)", p.dk);
      *chunked = false;
      return GDN_OK;
    case GDN_ALGO_CHUNKED:
      if (!can_chunk)
        return fail(GDN_EUNSUPPORTED, "chunked scan needs bf16 q/k/v with dk == dv == 128 (dk=%d dv=%d dtype=%d)",
                    p.dk, p.dv, (int)p.qkv_dtype);
      *chunked = true;
      return GDN_OK;
    case GDN_ALGO_AUTO: {
      // The chunked form pays off once sequences are several chunks long.
      const int64_t avg = p.n_tokens / p.n_seqs;
      *chunked = can_chunk && avg >= 128;
      if (!*chunked && !can_serial)
        return fail(GDN_EUNSUPPORTED, "no kernel for dk=%d (serial needs dk %% 4 == 0 and dk <= 256)", p.dk);
      return GDN_OK;
    }
  }
  return fail(GDN_EINVAL, "bad algo %d", (int)a->algo);
}

}  // namespace

namespace gdn {
gdn_status set_error(gdn_status st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return st;
}
// Base and size of the device allocation holding ptr (cuMemGetAddressRange,
// reached through the runtime's driver entry point).
gdn_status allocation_range(const void* ptr, void** base, size_t* size) {
  using GetRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static GetRange fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !f)
      return set_error(GDN_ECUDA, "cuMemGetAddressRange is not available");
    fn = reinterpret_cast<GetRange>(f);
  }
  CUdeviceptr b = 0;
  size_t n = 0;
  const CUresult r = fn(&b, &n, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return set_error(GDN_EINVAL, "cuMemGetAddressRange failed (%d): not a device allocation", (int)r);
  *base = reinterpret_cast<void*>(b);
  *size = n;
  return GDN_OK;
}
}  // namespace gdn

extern "C" {

int gdn_version(void) { return GDN_API_VERSION; }

const char* gdn_last_error(void) { return g_last_error.c_str(); }

gdn_status gdn_scan_workspace_size(const gdn_scan_args* args, size_t* bytes) {
  if (!bytes) return fail(GDN_EINVAL, "bytes is NULL");
  gdn::ScanParams p;
  gdn_status st = check_scan(args, &p, args ? args->n_seqs : 0);
  if (st != GDN_OK) return st;
  bool chunked = false;
  st = pick_algo(args, p, &chunked);
  if (st != GDN_OK) return st;
  *bytes = chunked ? gdn::chunked_workspace_bytes(p) : 0;
  return GDN_OK;
}

gdn_status gdn_scan(const gdn_scan_args* args, gdn_stream_t stream) {
  gdn::ScanParams p;
  gdn_status st = check_scan(args, &p, args ? args->n_seqs : 0);
  if (st != GDN_OK) return st;
  bool chunked = false;
  st = pick_algo(args, p, &chunked);
  if (st != GDN_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (chunked) {
    const size_t need = gdn::chunked_workspace_bytes(p);
    if (args->workspace_bytes < need || (need && !args->workspace))
      return fail(GDN_EINVAL, "workspace too small: %zu bytes given, %zu needed", args->workspace_bytes, need);
    return cuda_status(gdn::launch_chunked_scan(p, s), "chunked scan launch");
  }
  return cuda_status(gdn::launch_serial_scan(p, s), "serial scan launch");
}

gdn_status gdn_scan_gathered(const gdn_scan_args* args, const gdn_gather_args* gather, gdn_stream_t stream) {
  if (!gather) return fail(GDN_EINVAL, "gather is NULL");
  gdn::ScanParams p;
  gdn_status st = check_scan(args, &p, args ? args->n_seqs : 0);
  if (st != GDN_OK) return st;
  if (gather->hv_total < args->hv || gather->head0 < 0 || gather->head0 > gather->hv_total - args->hv)
    return fail(GDN_EINVAL, "heads [head0, head0 + hv) = [%d, %d) must lie in [0, hv_total = %d)", gather->head0,
                gather->head0 + args->hv, gather->hv_total);
  if (gather->n_peers < 0 || gather->n_peers > GDN_MAX_GATHER_PEERS)
    return fail(GDN_EINVAL, "n_peers must be in [0, %d] (got %d)", GDN_MAX_GATHER_PEERS, gather->n_peers);
  if (gather->reserved) return fail(GDN_EINVAL, "gather->reserved must be 0");
  if (!aligned16(args->out)) return fail(GDN_EINVAL, "out must be 16-byte aligned");
  for (int j = 0; j < gather->n_peers; ++j)
    if (!gather->peer_out[j] || !aligned16(gather->peer_out[j]) || gather->peer_out[j] == args->out)
      return fail(GDN_EINVAL, "peer_out[%d] must be a 16-byte aligned buffer other than out", j);
  bool chunked = false;
  st = pick_algo(args, p, &chunked);
  if (st != GDN_OK) return st;
  if (!chunked)
    return fail(GDN_EUNSUPPORTED, "the gathered scan runs on the chunked path only (bf16 q/k/v, dk == dv == 128, "
                                  "sequences of 128+ tokens on average or algo = CHUNKED)");
  const size_t need = gdn::chunked_workspace_bytes(p);
  if (args->workspace_bytes < need || (need && !args->workspace))
    return fail(GDN_EINVAL, "workspace too small: %zu bytes given, %zu needed", args->workspace_bytes, need);
  p.out_hv = gather->hv_total;
  p.head0 = gather->head0;
  p.n_peers = gather->n_peers;
  for (int j = 0; j < gather->n_peers; ++j) p.peer_out[j] = gather->peer_out[j];
  return cuda_status(gdn::launch_chunked_scan(p, static_cast<cudaStream_t>(stream)), "gathered scan launch");
}

gdn_status gdn_ipc_export(const void* ptr, unsigned char* handle, uint64_t* offset) {
  if (!ptr || !handle || !offset) return fail(GDN_EINVAL, "ptr, handle and offset must be non-NULL");
  void* base = nullptr;
  size_t size = 0;
  gdn_status st = gdn::allocation_range(ptr, &base, &size);
  if (st != GDN_OK) return st;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, base);
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == GDN_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = (uint64_t)(static_cast<const char*>(ptr) - static_cast<const char*>(base));
  return GDN_OK;
}

gdn_status gdn_ipc_import(const unsigned char* handle, uint64_t offset, void** ptr) {
  if (!handle || !ptr) return fail(GDN_EINVAL, "handle and ptr must be non-NULL");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcOpenMemHandle");
  *ptr = static_cast<char*>(base) + offset;
  return GDN_OK;
}

gdn_status gdn_ipc_release(void* ptr, uint64_t offset) {
  if (!ptr) return fail(GDN_EINVAL, "ptr is NULL");
  return cuda_status(cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset), "cudaIpcCloseMemHandle");
}

gdn_status gdn_decode(const gdn_decode_args* args, gdn_stream_t stream) {
  if (!args) return fail(GDN_EINVAL, "args is NULL");
  const gdn_scan_args* a = &args->base;
  if (a->cu_seqlens) return fail(GDN_EINVAL, "decode takes one token per sequence: cu_seqlens must be NULL");
  if (a->n_tokens != a->n_seqs)
    return fail(GDN_EINVAL, "decode takes one token per sequence: n_tokens (%lld) != n_seqs (%lld)",
                (long long)a->n_tokens, (long long)a->n_seqs);
  if (args->state_slots && args->n_slots <= 0) return fail(GDN_EINVAL, "n_slots must be > 0 with state_slots");
  gdn::ScanParams p;
  gdn_status st = check_scan(a, &p, args->state_slots ? args->n_slots : a->n_seqs);
  if (st != GDN_OK) return st;
  if (!gdn::serial_supported(p.dk))
    return fail(GDN_EUNSUPPORTED, "decode needs dk %% 4 == 0 and dk <= 256 (dk=%d)", p.dk);
  p.state_slots = args->state_slots;
  return cuda_status(gdn::launch_decode(p, static_cast<cudaStream_t>(stream)), "decode launch");
}

gdn_status gdn_forget_gate(const void* a, gdn_dtype a_dtype, int64_t a_stride_t, int64_t n, int32_t hv,
                           const float* A_log, const float* dt_bias, float* g, gdn_gate_kind kind,
                           gdn_stream_t stream) {
  if (n < 0 || hv <= 0) return fail(GDN_EINVAL, "forget_gate needs n >= 0 and hv > 0");
  if (!valid_dtype(a_dtype)) return fail(GDN_EINVAL, "bad a_dtype");
  if (kind != GDN_GATE_MULT && kind != GDN_GATE_LOG) return fail(GDN_EINVAL, "bad gate kind");
  if (a_stride_t < hv) return fail(GDN_EINVAL, "a_stride_t must be >= hv");
  if (n > 0 && (!a || !A_log || !dt_bias || !g)) return fail(GDN_EINVAL, "NULL pointer");
  return cuda_status(gdn::launch_forget_gate(a, a_dtype, a_stride_t, n, hv, A_log, dt_bias, g, kind,
                                             static_cast<cudaStream_t>(stream)),
                     "forget_gate launch");
}

}  // extern "C"

namespace {

struct BlockLayout {
  size_t q, k, v, g, beta, y, scan, total;
};

gdn_status check_block(const gdn_block_args* a, gdn::BlockParams* p, gdn::ScanParams* sp, BlockLayout* L,
                       bool* chunked) {
  if (!a) return fail(GDN_EINVAL, "args is NULL");
  if (a->hk <= 0 || a->hv <= 0 || a->dk <= 0 || a->dv <= 0 || a->hv % a->hk)
    return fail(GDN_EINVAL, "bad head shape (hk=%d hv=%d dk=%d dv=%d)", a->hk, a->hv, a->dk, a->dv);
  if (a->conv_kernel < 1 || a->conv_kernel > 8)
    return fail(a->conv_kernel < 1 ? GDN_EINVAL : GDN_EUNSUPPORTED, "conv_kernel must be in [1, 8] (got %d)",
                a->conv_kernel);
  if (a->dk > 256 || a->dv > 256) return fail(GDN_EUNSUPPORTED, "fused block supports head dims up to 256");
  if (a->n_tokens < 0 || a->n_seqs <= 0) return fail(GDN_EINVAL, "n_tokens must be >= 0 and n_seqs > 0");
  if (!a->cu_seqlens && a->n_tokens % a->n_seqs)
    return fail(GDN_EINVAL, "without cu_seqlens, n_tokens must be a multiple of n_seqs");
  if (a->act_dtype != GDN_F32 && a->act_dtype != GDN_BF16)
    return fail(GDN_EUNSUPPORTED, "act_dtype must be F32 or BF16");
  if (a->conv_state_dtype != GDN_F32 && a->conv_state_dtype != GDN_BF16)
    return fail(GDN_EUNSUPPORTED, "conv_state_dtype must be F32 or BF16");
  const int64_t width = 2LL * a->hk * a->dk + 2LL * a->hv * a->dv + 2LL * a->hv;
  if (a->mixed_stride_t < width)
    return fail(GDN_EINVAL, "mixed_stride_t (%lld) must be >= the row width %lld", (long long)a->mixed_stride_t,
                (long long)width);
  if (a->n_tokens > 0 && (!a->mixed || !a->out)) return fail(GDN_EINVAL, "mixed and out must be non-NULL");
  if (!a->conv_w || !a->A_log || !a->dt_bias || !a->norm_w || !a->state_out)
    return fail(GDN_EINVAL, "conv_w, A_log, dt_bias, norm_w and state_out must be non-NULL");
  if (a->conv_kernel > 1 && !a->conv_state_out) return fail(GDN_EINVAL, "conv_state_out must be non-NULL");
  if (!(a->eps >= 0.f)) return fail(GDN_EINVAL, "eps must be >= 0");

  const int64_t N = a->n_tokens;
  const size_t es = dtype_size(a->act_dtype);
  L->q = 0;
  L->k = round_up(L->q + (size_t)N * a->hk * a->dk * es, 256);
  L->v = round_up(L->k + (size_t)N * a->hk * a->dk * es, 256);
  L->g = round_up(L->v + (size_t)N * a->hv * a->dv * es, 256);
  L->beta = round_up(L->g + (size_t)N * a->hv * 4, 256);
  L->y = round_up(L->beta + (size_t)N * a->hv * 4, 256);
  L->scan = round_up(L->y + (size_t)N * a->hv * a->dv * es, 256);

  char* ws = static_cast<char*>(a->workspace);
  p->n_tokens = N;
  p->n_seqs = a->n_seqs;
  p->cu_seqlens = a->cu_seqlens;
  p->hk = a->hk;
  p->hv = a->hv;
  p->dk = a->dk;
  p->dv = a->dv;
  p->kernel = a->conv_kernel;
  p->mixed = a->mixed;
  p->mixed_st = a->mixed_stride_t;
  p->act_dtype = a->act_dtype;
  p->conv_w = a->conv_w;
  p->conv_state_in = a->conv_state_in;
  p->conv_state_out = a->conv_state_out;
  p->conv_state_dtype = a->conv_state_dtype;
  p->A_log = a->A_log;
  p->dt_bias = a->dt_bias;
  p->norm_w = a->norm_w;
  p->eps = a->eps;
  p->q = ws + L->q;
  p->k = ws + L->k;
  p->v = ws + L->v;
  p->g_log = reinterpret_cast<float*>(ws + L->g);
  p->beta = reinterpret_cast<float*>(ws + L->beta);
  p->y = ws + L->y;
  p->out = a->out;

  gdn_scan_args sa = {};
  sa.n_tokens = N;
  sa.n_seqs = a->n_seqs;
  sa.cu_seqlens = a->cu_seqlens;
  sa.hk = a->hk;
  sa.hv = a->hv;
  sa.dk = a->dk;
  sa.dv = a->dv;
  sa.q = p->q;
  sa.q_stride_t = (int64_t)a->hk * a->dk;
  sa.q_stride_h = a->dk;
  sa.k = p->k;
  sa.k_stride_t = (int64_t)a->hk * a->dk;
  sa.k_stride_h = a->dk;
  sa.v = p->v;
  sa.v_stride_t = (int64_t)a->hv * a->dv;
  sa.v_stride_h = a->dv;
  sa.g = p->g_log;
  sa.g_stride_t = a->hv;
  sa.beta = p->beta;
  sa.beta_stride_t = a->hv;
  sa.state_in = a->state_in;
  sa.state_out = a->state_out;
  sa.out = p->y;
  sa.qkv_dtype = a->act_dtype;
  sa.gate_dtype = GDN_F32;
  sa.out_dtype = a->act_dtype;  // y rounded to the act dtype, as the reference does before the norm
  sa.gate_kind = GDN_GATE_LOG;
  sa.algo = a->algo;
  gdn_status st = check_scan(&sa, sp, a->n_seqs, /*check_pointers=*/false);
  if (st != GDN_OK) return st;
  st = pick_algo(&sa, *sp, chunked);
  if (st != GDN_OK) return st;
  // The chunked scan applies the gated norm in its output stage and writes the
  // layer output directly (bf16 activations, z 16-byte aligned).
  const int64_t conv_dim = 2LL * a->hk * a->dk + (int64_t)a->hv * a->dv;
  if (*chunked && a->act_dtype == GDN_BF16 && a->mixed_stride_t % 8 == 0 && conv_dim % 8 == 0 &&
      aligned16(a->mixed)) {
    sp->z = static_cast<const __nv_bfloat16*>(a->mixed) + conv_dim;
    sp->z_st = a->mixed_stride_t;
    sp->norm_w = a->norm_w;
    sp->norm_eps = a->eps;
    sp->out = a->out;
  }
  const size_t scan_bytes = *chunked ? gdn::chunked_workspace_bytes(*sp) : 0;
  L->total = L->scan + scan_bytes;
  sp->workspace = ws + L->scan;
  sp->workspace_bytes = scan_bytes;
  return GDN_OK;
}

}  // namespace

extern "C" {

gdn_status gdn_block_workspace_size(const gdn_block_args* args, size_t* bytes) {
  if (!bytes) return fail(GDN_EINVAL, "bytes is NULL");
  gdn::BlockParams p;
  gdn::ScanParams sp;
  BlockLayout L;
  bool chunked = false;
  gdn_status st = check_block(args, &p, &sp, &L, &chunked);
  if (st != GDN_OK) return st;
  *bytes = L.total;
  return GDN_OK;
}

gdn_status gdn_fused_block(const gdn_block_args* args, gdn_stream_t stream) {
  gdn::BlockParams p;
  gdn::ScanParams sp;
  BlockLayout L;
  bool chunked = false;
  gdn_status st = check_block(args, &p, &sp, &L, &chunked);
  if (st != GDN_OK) return st;
  if (args->workspace_bytes < L.total || (L.total && !args->workspace))
    return fail(GDN_EINVAL, "workspace too small: %zu bytes given, %zu needed", args->workspace_bytes, L.total);
  if (!aligned16(args->workspace)) return fail(GDN_EINVAL, "workspace must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!chunked && gdn::block_decode_supported(p, sp.state_in, sp.state_out))  // one token per sequence
    return cuda_status(gdn::launch_block_decode(p, sp.state_in, sp.state_out, s), "block decode launch");
  st = cuda_status(gdn::launch_block_prologue(p, s), "block prologue launch");
  if (st != GDN_OK) return st;
  st = cuda_status(gdn::launch_block_conv_tail(p, s), "conv tail launch");
  if (st != GDN_OK) return st;
  st = cuda_status(chunked ? gdn::launch_chunked_scan(sp, s) : gdn::launch_serial_scan(sp, s), "scan launch");
  if (st != GDN_OK) return st;
  if (sp.z) return GDN_OK;  // the scan's output stage did the gated norm
  return cuda_status(gdn::launch_block_epilogue(p, s), "block epilogue launch");
}

gdn_status gdn_test_set_wait_limit(uint64_t ns) {
  unsigned long long cur = 0;
  int fault = 0;
  cudaError_t e = gdn::read_test_hooks(&cur, &fault);
  if (e == cudaSuccess) e = gdn::set_test_hooks(ns, fault);
  return cuda_status(e, "setting the wait limit");
}

gdn_status gdn_test_inject_fault(int32_t fault) {
  if (fault < 0 || fault > 1) return fail(GDN_EINVAL, "unknown test fault %d", (int)fault);
  unsigned long long cur = 0;
  int old = 0;
  cudaError_t e = gdn::read_test_hooks(&cur, &old);
  if (e == cudaSuccess) e = gdn::set_test_hooks(cur, fault);
  return cuda_status(e, "setting the test fault");
}

gdn_status gdn_check_device_errors(gdn_stream_t stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_status(e, "stream synchronize");
  unsigned code = 0;
  e = gdn::read_and_clear_device_error(&code);
  if (e == cudaSuccess) {
    unsigned code2 = 0;
    e = gdn::read_and_clear_qlinear_error(&code2);
    code |= code2;
  }
  if (e == cudaSuccess) {
    unsigned code3 = 0;
    e = gdn::read_and_clear_attn_error(&code3);
    code |= code3;
  }
  if (e != cudaSuccess) return cuda_status(e, "reading the device error word");
  if (code) return fail(GDN_ETIMEOUT, "a bounded device wait gave up (code 0x%x)", code);
  return GDN_OK;
}

}  // extern "C"
