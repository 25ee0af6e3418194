// C ABI of libminiep_b200: context, symmetric buffers, placement tables,
// and the layer-step entry points. See include/miniep_b200.h.
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "miniep_b200.h"
#include "mep_internal.h"

using namespace mep;

struct mep_ctx {
  int rank = 0, world = 1, device = 0, L = 0, E = 0, k = 0, H = 0, I = 0, dtype = 0;
  int64_t max_tokens = 0, cap_rows = 0;
  int num_sms = 0;
  size_t elt = 4;
  // symmetric region (exported over CUDA IPC): flags | counts | meta | land | ret
  uint8_t* sym = nullptr;
  size_t sym_bytes = 0, off_flags = 0, off_cnt = 0, off_meta = 0, off_land = 0, off_ret = 0;
  void* recv_x = nullptr;  // expert-grouped receive rows (local only)
  uint8_t* peer_base[kMaxWorld] = {};
  bool peer_open[kMaxWorld] = {};
  PeerPtrs peers{};
  // local buffers
  void* act = nullptr;
  int32_t* chunk_hist = nullptr;
  int32_t* ent_dest = nullptr;
  int32_t* ent_grp = nullptr;
  int32_t* my_counts = nullptr;
  Layout* layout = nullptr;
  int32_t* owners = nullptr;  // [L][E][kMaxWorld]
  int32_t* nrep = nullptr;    // [L][E]
  int64_t* rr = nullptr;      // [L][E]
  int64_t* route_counts = nullptr;    // [L][E]
  int64_t* recv_per_layer = nullptr;  // [L]
  unsigned int* done_ctr = nullptr;   // kDoneCounters completion counters (mep_internal.h)
  int* err_host = nullptr;
  int* err_dev = nullptr;
  uint32_t* seq = nullptr;  // device: sequence number of the current layer step
  uint64_t* tl = nullptr;   // device: step timeline stamps (MEP_TL_SLOTS)
  int tl_on = 0;            // pass tl to the kernels (option "timeline")
  unsigned long long timeout_ns = 10ull * 1000 * 1000 * 1000;
  int force_simt = 0;
  int tc_single_cta = 0;
  int dispatch_per_warp = 1;  // 0: the streaming engine (k_dispatch_stream) instead of one warp per token
  int router_no_tc = 0;       // 1: never the tcgen05 router
  int ffn_ast = 0;            // 1: A-stationary GEMM2 (measured slower: a shallower B ring)
  int ffn_prefetch = 0;       // 1: the GEMMs prefetch their next tile's A rows into L2 (measured slower)
  std::vector<int> placed, n_local_l;
  int cur_layer = -1, stage = 0;
  int64_t cur_n = 0;
  std::string err;
};

namespace {

thread_local std::string g_create_err;

int fail(mep_ctx* c, int code, const std::string& msg) {
  if (c)
    c->err = msg;
  else
    g_create_err = msg;
  return code;
}

int cuda_fail(mep_ctx* c, cudaError_t e, const char* what) {
  return fail(c, MEP_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define MEP_CK(c, call)                                      \
  do {                                                       \
    cudaError_t e_ = (call);                                 \
    if (e_ != cudaSuccess) return cuda_fail((c), e_, #call); \
  } while (0)

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

void build_peers(mep_ctx* c) {
  for (int r = 0; r < kMaxWorld; ++r) {
    uint8_t* b = r < c->world ? c->peer_base[r] : nullptr;
    c->peers.land[r] = b ? b + c->off_land : nullptr;
    c->peers.recv_x[r] = r == c->rank ? c->recv_x : nullptr;  // only this rank's rows are stored here
    c->peers.recv_meta[r] = b ? reinterpret_cast<int32_t*>(b + c->off_meta) : nullptr;
    c->peers.ret[r] = b ? b + c->off_ret : nullptr;
    c->peers.cnt_in[r] = b ? reinterpret_cast<int32_t*>(b + c->off_cnt) : nullptr;
    c->peers.flags[r] = b ? reinterpret_cast<uint32_t*>(b + c->off_flags) : nullptr;
  }
}

WaitCfg wait_cfg(const mep_ctx* c) { return WaitCfg{c->err_dev, c->timeout_ns}; }

uint64_t* tl_of(const mep_ctx* c) { return c->tl_on ? c->tl : nullptr; }

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

int use_device(mep_ctx* c) {
  int cur = -1;
  MEP_CK(c, cudaGetDevice(&cur));
  if (cur != c->device) MEP_CK(c, cudaSetDevice(c->device));
  return MEP_OK;
}

int check_layer(mep_ctx* c, int layer) {
  if (layer < 0 || layer >= c->L) return fail(c, MEP_ERR_INVALID, "layer out of range");
  if (!c->placed[layer])
    return fail(c, MEP_ERR_STATE, "mep_set_placement was not called for layer " +
                                      std::to_string(layer));
  return MEP_OK;
}

int check_peers(mep_ctx* c) {
  for (int r = 0; r < c->world; ++r)
    if (!c->peer_base[r])
      return fail(c, MEP_ERR_STATE, "peer " + std::to_string(r) +
                                        " buffers not opened (mep_ipc_open)");
  return MEP_OK;
}

const int32_t* owners_of(const mep_ctx* c, int layer) {
  return c->owners + (int64_t)layer * c->E * kMaxWorld;
}
const int32_t* nrep_of(const mep_ctx* c, int layer) { return c->nrep + (int64_t)layer * c->E; }

}  // namespace

namespace mep {
// Message for mep_last_error(NULL), set by entry points that take no context.
void set_global_error(const std::string& msg) { g_create_err = msg; }
}  // namespace mep

extern "C" {

int mep_version(void) { return 100; }

const char* mep_last_error(const mep_ctx* ctx) {
  return ctx ? ctx->err.c_str() : g_create_err.c_str();
}

int mep_ctx_create(int rank, int world, int device, int num_layers, int num_experts, int topk,
                   int hidden, int inter, int64_t max_tokens, int dtype,
                   int64_t recv_capacity_rows, mep_ctx** out) {
  if (!out) return fail(nullptr, MEP_ERR_INVALID, "out is NULL");
  *out = nullptr;
  if (world < 1 || world > kMaxWorld) return fail(nullptr, MEP_ERR_INVALID, "world must be 1..8");
  if (rank < 0 || rank >= world) return fail(nullptr, MEP_ERR_INVALID, "rank out of range");
  if (num_layers < 1) return fail(nullptr, MEP_ERR_INVALID, "num_layers must be >= 1");
  if (num_experts < 1 || num_experts > kMaxExperts)
    return fail(nullptr, MEP_ERR_INVALID, "num_experts must be 1..128");
  if (topk < 1 || topk > kMaxTopk || topk > num_experts)
    return fail(nullptr, MEP_ERR_INVALID, "topk must be 1..min(16, E)");
  if (dtype != MEP_F32 && dtype != MEP_BF16) return fail(nullptr, MEP_ERR_INVALID, "bad dtype");
  const size_t elt = dtype == MEP_BF16 ? 2 : 4;
  if (hidden < 1 || (hidden * elt) % 16 != 0)
    return fail(nullptr, MEP_ERR_INVALID, "hidden * element size must be a multiple of 16 bytes");
  if (hidden % 64 != 0 || inter < 32 || inter % 32 != 0)
    return fail(nullptr, MEP_ERR_INVALID, "hidden must be a multiple of 64, inter of 32");
  if (max_tokens < 1 || max_tokens * topk >= (int64_t(1) << 24))
    return fail(nullptr, MEP_ERR_INVALID, "max_tokens * topk must be in [1, 2^24)");

  mep_ctx* c = new mep_ctx();
  c->rank = rank;
  c->world = world;
  c->device = device;
  c->L = num_layers;
  c->E = num_experts;
  c->k = topk;
  c->H = hidden;
  c->I = inter;
  c->dtype = dtype;
  c->elt = elt;
  c->max_tokens = max_tokens;
  c->cap_rows = recv_capacity_rows > 0
                    ? recv_capacity_rows
                    : (int64_t)world * max_tokens * topk + (int64_t)num_experts * kRowAlign;
  c->placed.assign(num_layers, 0);
  c->n_local_l.assign(num_layers, 0);
  auto bail = [&](int rc) {
    g_create_err = c->err;
    mep_ctx_destroy(c);
    return rc;
  };
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return bail(cuda_fail(c, e, "cudaSetDevice"));
  e = cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return bail(cuda_fail(c, e, "cudaDeviceGetAttribute"));

  size_t off = 0;
  c->off_flags = off;
  off = align_up(off + 4 * kMaxWorld * sizeof(uint32_t), 1024);
  c->off_cnt = off;
  off = align_up(off + (size_t)kMaxWorld * kMaxWorld * kMaxExperts * sizeof(int32_t), 1024);
  c->off_meta = off;
  off = align_up(off + (size_t)c->cap_rows * sizeof(int32_t), 1024);
  c->off_land = off;  // [src rank][max_tokens][H]: each token row once per destination rank
  off = align_up(off + (size_t)(world > 1 ? world : 0) * max_tokens * hidden * elt, 1024);
  c->off_ret = off;  // return rows: one per entry of this rank's tokens
  off = align_up(off + (size_t)max_tokens * topk * hidden * elt, 1024);
  c->sym_bytes = off;

  const int64_t max_entries = max_tokens * topk;
  const int64_t nchunks = (max_entries + kRouteChunkTokens - 1) / kRouteChunkTokens;
  struct {
    void** p;
    size_t bytes;
  } allocs[] = {
      {reinterpret_cast<void**>(&c->sym), c->sym_bytes},
      {&c->act, (size_t)c->cap_rows * inter * elt},
      {&c->recv_x, (size_t)c->cap_rows * hidden * elt},
      {reinterpret_cast<void**>(&c->chunk_hist), (size_t)nchunks * num_experts * 4},
      {reinterpret_cast<void**>(&c->ent_dest), (size_t)max_entries * 4},
      {reinterpret_cast<void**>(&c->ent_grp), (size_t)max_entries * 4},
      {reinterpret_cast<void**>(&c->my_counts), (size_t)kMaxWorld * kMaxExperts * 4},
      {reinterpret_cast<void**>(&c->layout), sizeof(Layout)},
      {reinterpret_cast<void**>(&c->owners), (size_t)num_layers * num_experts * kMaxWorld * 4},
      {reinterpret_cast<void**>(&c->nrep), (size_t)num_layers * num_experts * 4},
      {reinterpret_cast<void**>(&c->rr), (size_t)num_layers * num_experts * 8},
      {reinterpret_cast<void**>(&c->route_counts), (size_t)num_layers * num_experts * 8},
      {reinterpret_cast<void**>(&c->recv_per_layer), (size_t)num_layers * 8},
      {reinterpret_cast<void**>(&c->done_ctr), kDoneCounters * sizeof(unsigned int)},
      {reinterpret_cast<void**>(&c->seq), 2 * sizeof(uint32_t)},  // [0] layer step, [1] barrier
      {reinterpret_cast<void**>(&c->tl), (size_t)kTlSlots * sizeof(uint64_t)},
  };
  for (auto& a : allocs) {
    e = cudaMalloc(a.p, a.bytes);
    if (e != cudaSuccess) return bail(cuda_fail(c, e, "cudaMalloc"));
    e = cudaMemset(*a.p, 0, a.bytes);
    if (e != cudaSuccess) return bail(cuda_fail(c, e, "cudaMemset"));
  }
  e = cudaHostAlloc(reinterpret_cast<void**>(&c->err_host), sizeof(int), cudaHostAllocMapped);
  if (e != cudaSuccess) return bail(cuda_fail(c, e, "cudaHostAlloc"));
  *c->err_host = 0;
  e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->err_dev), c->err_host, 0);
  if (e != cudaSuccess) return bail(cuda_fail(c, e, "cudaHostGetDevicePointer"));
  e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return bail(cuda_fail(c, e, "cudaDeviceSynchronize"));
  c->peer_base[rank] = c->sym;
  build_peers(c);
  *out = c;
  return MEP_OK;
}

int mep_ctx_destroy(mep_ctx* c) {
  if (!c) return MEP_OK;
  int cur = -1;
  if (cudaGetDevice(&cur) == cudaSuccess && cur != c->device) cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < kMaxWorld; ++r)
    if (c->peer_open[r] && c->peer_base[r]) cudaIpcCloseMemHandle(c->peer_base[r]);
  void* ptrs[] = {c->sym,      c->act,    c->recv_x,     c->chunk_hist,   c->ent_dest,     c->ent_grp,
                  c->my_counts, c->layout, c->owners,     c->nrep,         c->rr,
                  c->route_counts, c->recv_per_layer, c->done_ctr, c->seq, c->tl};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  if (c->err_host) cudaFreeHost(c->err_host);
  if (cur >= 0 && cur != c->device) cudaSetDevice(cur);
  delete c;
  return MEP_OK;
}

int mep_ipc_handle(mep_ctx* c, void* handle_out) {
  if (!c || !handle_out) return fail(c, MEP_ERR_INVALID, "NULL argument");
  if (int rc = use_device(c)) return rc;
  cudaIpcMemHandle_t h;
  MEP_CK(c, cudaIpcGetMemHandle(&h, c->sym));
  static_assert(sizeof(h) == MEP_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  return MEP_OK;
}

int mep_ipc_open(mep_ctx* c, int peer, const void* handle) {
  if (!c || !handle) return fail(c, MEP_ERR_INVALID, "NULL argument");
  if (peer < 0 || peer >= c->world) return fail(c, MEP_ERR_INVALID, "peer out of range");
  if (peer == c->rank) return MEP_OK;
  if (c->peer_open[peer]) return fail(c, MEP_ERR_STATE, "peer already opened");
  if (int rc = use_device(c)) return rc;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  MEP_CK(c, cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  c->peer_base[peer] = static_cast<uint8_t*>(p);
  c->peer_open[peer] = true;
  build_peers(c);
  return MEP_OK;
}

int mep_set_placement(mep_ctx* c, int layer, const int64_t* table, const int64_t* n_rep,
                      int rmax) {
  if (!c || !table || !n_rep) return fail(c, MEP_ERR_INVALID, "NULL argument");
  if (layer < 0 || layer >= c->L) return fail(c, MEP_ERR_INVALID, "layer out of range");
  if (rmax < 1) return fail(c, MEP_ERR_INVALID, "rmax must be >= 1");
  std::vector<int32_t> own((size_t)c->E * kMaxWorld), nr(c->E);
  int n_local = 0;
  for (int e = 0; e < c->E; ++e) {
    const int64_t n = n_rep[e];
    if (n < 1 || n > rmax || n > c->world)
      return fail(c, MEP_ERR_INVALID, "expert " + std::to_string(e) + ": n_rep out of range");
    bool mine = false;
    for (int j = 0; j < n; ++j) {
      const int64_t r = table[(int64_t)e * rmax + j];
      if (r < 0 || r >= c->world)
        return fail(c, MEP_ERR_INVALID, "expert " + std::to_string(e) + ": owner rank out of range");
      for (int i = 0; i < j; ++i)
        if (own[(size_t)e * kMaxWorld + i] == r)
          return fail(c, MEP_ERR_INVALID, "expert " + std::to_string(e) + ": duplicate owner");
      own[(size_t)e * kMaxWorld + j] = (int32_t)r;
      mine |= r == c->rank;
    }
    for (int j = (int)n; j < kMaxWorld; ++j) own[(size_t)e * kMaxWorld + j] = own[(size_t)e * kMaxWorld];
    nr[e] = (int32_t)n;
    n_local += mine;
  }
  if (int rc = use_device(c)) return rc;
  MEP_CK(c, cudaMemcpy(c->owners + (int64_t)layer * c->E * kMaxWorld, own.data(),
                       own.size() * 4, cudaMemcpyHostToDevice));
  MEP_CK(c, cudaMemcpy(c->nrep + (int64_t)layer * c->E, nr.data(), nr.size() * 4,
                       cudaMemcpyHostToDevice));
  c->placed[layer] = 1;
  c->n_local_l[layer] = n_local;
  return MEP_OK;
}

int mep_reset_rr(mep_ctx* c, void* stream) {
  if (!c) return MEP_ERR_INVALID;
  if (int rc = use_device(c)) return rc;
  MEP_CK(c, cudaMemsetAsync(c->rr, 0, (size_t)c->L * c->E * 8, as_stream(stream)));
  return MEP_OK;
}

int mep_dest_ranks(mep_ctx* c, int layer, const int64_t* expert_ids, int64_t m,
                   int64_t* dest_out, void* stream) {
  if (!c) return MEP_ERR_INVALID;
  if (int rc = check_layer(c, layer)) return rc;
  if (m < 0 || m > c->max_tokens * c->k)
    return fail(c, MEP_ERR_INVALID, "m must be in [0, max_tokens * topk]");
  if (m > 0 && (!expert_ids || !dest_out)) return fail(c, MEP_ERR_INVALID, "NULL argument");
  if (int rc = use_device(c)) return rc;
  launch_dest_only(m, c->E, expert_ids, owners_of(c, layer), nrep_of(c, layer),
                   c->rr + (int64_t)layer * c->E, c->chunk_hist, c->ent_dest, c->ent_grp,
                   dest_out, wait_cfg(c), as_stream(stream));
  MEP_CK(c, cudaGetLastError());
  return MEP_OK;
}

int mep_router_topk(mep_ctx* c, const void* x, const void* router_w, const float* bias, int64_t n,
                    int64_t* topk_idx_out, void* topk_gate_out, float* logits_out, void* stream) {
  if (!c) return MEP_ERR_INVALID;
  if (n < 0) return fail(c, MEP_ERR_INVALID, "n < 0");
  if (n > 0 && (!x || !router_w || !topk_idx_out || !topk_gate_out))
    return fail(c, MEP_ERR_INVALID, "NULL argument");
  if (int rc = use_device(c)) return rc;
  launch_router(c->dtype, x, router_w, bias, n, c->H, c->E, c->k, topk_idx_out, topk_gate_out,
                logits_out, c->num_sms, !c->router_no_tc, c->err_dev, tl_of(c), as_stream(stream));
  MEP_CK(c, cudaGetLastError());
  return MEP_OK;
}

int mep_route(mep_ctx* c, int layer, const int64_t* topk_idx, const uint8_t* valid, int64_t n,
              int n_local, void* stream) {
  if (!c) return MEP_ERR_INVALID;
  if (int rc = check_layer(c, layer)) return rc;
  if (n < 0 || n > c->max_tokens) return fail(c, MEP_ERR_INVALID, "n must be in [0, max_tokens]");
  if (n > 0 && !topk_idx) return fail(c, MEP_ERR_INVALID, "topk_idx is NULL");
  if (n_local != c->n_local_l[layer])
    return fail(c, MEP_ERR_INVALID,
                "n_local " + std::to_string(n_local) + " does not match the placement (" +
                    std::to_string(c->n_local_l[layer]) + " experts resident on this rank)");
  if (int rc = check_peers(c)) return rc;
  if (int rc = use_device(c)) return rc;
  c->cur_layer = layer;
  c->cur_n = n;
  launch_route(n, c->k, c->E, c->world, c->rank, topk_idx, valid, owners_of(c, layer),
               nrep_of(c, layer), c->rr + (int64_t)layer * c->E,
               c->route_counts + (int64_t)layer * c->E, c->chunk_hist, c->ent_dest, c->ent_grp,
               c->my_counts, c->peers, c->seq, c->done_ctr + 2, c->num_sms,
               reinterpret_cast<const int32_t*>(c->sym + c->off_cnt),
               reinterpret_cast<const uint32_t*>(c->sym + c->off_flags), c->recv_per_layer + layer,
               c->cap_rows, c->layout, wait_cfg(c), tl_of(c), as_stream(stream));
  MEP_CK(c, cudaGetLastError());
  c->stage = 1;
  return MEP_OK;
}

int mep_dispatch(mep_ctx* c, const void* x, const int64_t* topk_idx, int64_t n, void* stream) {
  if (!c) return MEP_ERR_INVALID;
  if (c->stage != 1) return fail(c, MEP_ERR_STATE, "mep_dispatch must follow mep_route");
  if (n != c->cur_n) return fail(c, MEP_ERR_INVALID, "n differs from the routed step");
  if (n > 0 && (!x || !topk_idx)) return fail(c, MEP_ERR_INVALID, "NULL argument");
  if (n > 0 && (reinterpret_cast<uintptr_t>(x) & 15u) != 0)  // rows are read in 16-byte pieces
    return fail(c, MEP_ERR_INVALID, "x must start on a 16-byte boundary");
  if (int rc = use_device(c)) return rc;
  // the receive layout was computed by mep_route's kernel
  launch_dispatch(c->dtype, n, c->k, c->H, c->world, c->rank, c->max_tokens,
                  x, topk_idx, c->ent_dest,
                  c->ent_grp, c->layout, c->peers, c->done_ctr, c->seq, c->num_sms,
                  c->dispatch_per_warp, c->err_dev, tl_of(c), as_stream(stream));
  // the stage ends when every rank's rows for this rank have landed and sit in
  // their expert-segment rows (one rank: stream order already says so)
  if (c->world > 1)
    launch_fanout(c->dtype, c->H, c->k, c->rank, c->world, c->max_tokens, c->layout,
                  reinterpret_cast<const int32_t*>(c->sym + c->off_meta), c->sym + c->off_land,
                  c->recv_x, reinterpret_cast<const uint32_t*>(c->sym + c->off_flags), c->seq,
                  wait_cfg(c), c->num_sms, tl_of(c), as_stream(stream));
  MEP_CK(c, cudaGetLastError());
  c->stage = 2;
  return MEP_OK;
}

int mep_expert_ffn(mep_ctx* c, const void* w_in, const void* w_out, int n_local, void* stream) {
  if (!c) return MEP_ERR_INVALID;
  if (c->stage != 2) return fail(c, MEP_ERR_STATE, "mep_expert_ffn must follow mep_dispatch");
  if (n_local != c->n_local_l[c->cur_layer])
    return fail(c, MEP_ERR_INVALID, "n_local does not match the placement");
  if (n_local > 0 && (!w_in || !w_out)) return fail(c, MEP_ERR_INVALID, "NULL weights");
  if (int rc = use_device(c)) return rc;
  FfnArgs a{};
  a.dtype = c->dtype;
  a.hidden = c->H;
  a.inter = c->I;
  a.world = c->world;
  a.rank = c->rank;
  a.cap_rows = c->cap_rows;
  a.recv_x = c->recv_x;
  a.ret_rows = c->max_tokens * c->k;
  a.act = c->act;
  a.w_in = w_in;
  a.w_out = w_out;
  a.layout = c->layout;
  a.peers = c->peers;
  a.done_ctr = c->done_ctr + 1;
  a.seq = c->seq;
  a.num_sms = c->num_sms;
  a.force_simt = c->force_simt;
  a.tc_single_cta = c->tc_single_cta;
  a.ast = c->ffn_ast;
  a.prefetch = c->ffn_prefetch;
  a.n_local_weights = n_local;
  a.err = c->err_dev;
  a.tl = tl_of(c);
  // a rank without resident experts still runs the (empty) kernel to signal
  // completion; give the tensor maps a valid base
  if (n_local == 0) {
    a.w_in = c->act;
    a.w_out = c->act;
  }
  const int rc = launch_ffn(a, as_stream(stream));
  if (rc > 0) return cuda_fail(c, static_cast<cudaError_t>(rc), "expert FFN launch");
  if (rc < 0) return fail(c, MEP_ERR_CUDA, "expert FFN set-up failed (code " + std::to_string(rc) + ")");
  c->stage = 3;
  return MEP_OK;
}

int mep_combine(mep_ctx* c, const void* topk_gate, const uint8_t* valid, int64_t n,
                const void* h, float residual_multiplier, void* out, void* h_out, void* stream) {
  if (!c) return MEP_ERR_INVALID;
  if (c->stage != 3) return fail(c, MEP_ERR_STATE, "mep_combine must follow mep_expert_ffn");
  if (n != c->cur_n) return fail(c, MEP_ERR_INVALID, "n differs from the routed step");
  if (n > 0 && !topk_gate) return fail(c, MEP_ERR_INVALID, "topk_gate is NULL");
  if (n > 0 && !out && !h_out) return fail(c, MEP_ERR_INVALID, "no output given");
  if (h_out && !h) return fail(c, MEP_ERR_INVALID, "h_out needs h");
  if (int rc = use_device(c)) return rc;
  // ent_grp holds each entry's return row since the dispatch
  launch_combine(c->dtype, n, c->k, c->H, c->world, c->sym + c->off_ret, c->ent_grp, topk_gate,
                 valid, h,
                 residual_multiplier, out, h_out,
                 reinterpret_cast<const uint32_t*>(c->sym + c->off_flags), c->seq, wait_cfg(c),
                 c->num_sms, tl_of(c), as_stream(stream));
  MEP_CK(c, cudaGetLastError());
  c->stage = 0;
  return MEP_OK;
}

int mep_moe_forward(mep_ctx* c, int layer, const void* x, const int64_t* topk_idx,
                    const void* topk_gate, const uint8_t* valid, int64_t n, const void* w_in,
                    const void* w_out, int n_local, void* out, void* stream) {
  int rc;
  if ((rc = mep_route(c, layer, topk_idx, valid, n, n_local, stream))) return rc;
  if ((rc = mep_dispatch(c, x, topk_idx, n, stream))) return rc;
  if ((rc = mep_expert_ffn(c, w_in, w_out, n_local, stream))) return rc;
  return mep_combine(c, topk_gate, valid, n, nullptr, 0.f, out, nullptr, stream);
}

int mep_moe_block(mep_ctx* c, int layer, const void* h, const void* x, const void* router_w,
                  const float* bias, const uint8_t* valid, int64_t n, const void* w_in,
                  const void* w_out, int n_local, float residual_multiplier, void* h_out,
                  int64_t* topk_idx_out, void* topk_gate_out, void* stream) {
  int rc;
  if (n > 0 && (!h || !h_out)) return fail(c, MEP_ERR_INVALID, "NULL argument");
  if ((rc = mep_router_topk(c, x, router_w, bias, n, topk_idx_out, topk_gate_out, nullptr,
                            stream)))
    return rc;
  if ((rc = mep_route(c, layer, topk_idx_out, valid, n, n_local, stream))) return rc;
  if ((rc = mep_dispatch(c, x, topk_idx_out, n, stream))) return rc;
  if ((rc = mep_expert_ffn(c, w_in, w_out, n_local, stream))) return rc;
  return mep_combine(c, topk_gate_out, valid, n, h, residual_multiplier, nullptr, h_out, stream);
}

int mep_rmsnorm(mep_ctx* c, const void* h, const void* w, float eps, int64_t n, void* x_out,
                void* stream) {
  if (!c) return MEP_ERR_INVALID;
  if (n < 0) return fail(c, MEP_ERR_INVALID, "n must be >= 0");
  if (n > 0 && (!h || !w || !x_out)) return fail(c, MEP_ERR_INVALID, "NULL argument");
  if (n > 0 && ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(w) |
                 reinterpret_cast<uintptr_t>(x_out)) & 15u) != 0)
    return fail(c, MEP_ERR_INVALID, "h, w and x_out must start on 16-byte boundaries");
  if (!(eps >= 0.f)) return fail(c, MEP_ERR_INVALID, "eps must be >= 0");
  if (int rc = use_device(c)) return rc;
  launch_rmsnorm(c->dtype, n, c->H, h, w, eps, x_out, tl_of(c), as_stream(stream));
  MEP_CK(c, cudaGetLastError());
  return MEP_OK;
}

int mep_moe_block_from_h(mep_ctx* c, int layer, const void* h, const void* norm_w, float eps,
                         const void* router_w, const float* bias, const uint8_t* valid,
                         int64_t n, const void* w_in, const void* w_out, int n_local,
                         float residual_multiplier, void* h_out, void* x_out,
                         int64_t* topk_idx_out, void* topk_gate_out, void* stream) {
  if (int rc = mep_rmsnorm(c, h, norm_w, eps, n, x_out, stream)) return rc;
  return mep_moe_block(c, layer, h, x_out, router_w, bias, valid, n, w_in, w_out, n_local,
                       residual_multiplier, h_out, topk_idx_out, topk_gate_out, stream);
}

int mep_read_stats(mep_ctx* c, int64_t* route_counts_out, int64_t* recv_out, void* stream) {
  if (!c) return MEP_ERR_INVALID;
  if (int rc = use_device(c)) return rc;
  cudaStream_t st = as_stream(stream);
  if (route_counts_out)
    MEP_CK(c, cudaMemcpyAsync(route_counts_out, c->route_counts, (size_t)c->L * c->E * 8,
                              cudaMemcpyDeviceToHost, st));
  if (recv_out)
    MEP_CK(c, cudaMemcpyAsync(recv_out, c->recv_per_layer, (size_t)c->L * 8,
                              cudaMemcpyDeviceToHost, st));
  MEP_CK(c, cudaStreamSynchronize(st));
  return MEP_OK;
}

int mep_reset_stats(mep_ctx* c, void* stream) {
  if (!c) return MEP_ERR_INVALID;
  if (int rc = use_device(c)) return rc;
  MEP_CK(c, cudaMemsetAsync(c->route_counts, 0, (size_t)c->L * c->E * 8, as_stream(stream)));
  MEP_CK(c, cudaMemsetAsync(c->recv_per_layer, 0, (size_t)c->L * 8, as_stream(stream)));
  return MEP_OK;
}

int mep_last_recv_rows(mep_ctx* c, int64_t* rows_out, void* stream) {
  if (!c || !rows_out) return fail(c, MEP_ERR_INVALID, "NULL argument");
  if (int rc = use_device(c)) return rc;
  int v = 0;
  MEP_CK(c, cudaMemcpyAsync(&v, &c->layout->recv_rows, sizeof(int), cudaMemcpyDeviceToHost,
                            as_stream(stream)));
  MEP_CK(c, cudaStreamSynchronize(as_stream(stream)));
  *rows_out = v;
  return MEP_OK;
}

int mep_check(mep_ctx* c) {
  if (!c) return MEP_ERR_INVALID;
  const int code = *(volatile int*)c->err_host;
  if (code == kErrNone) return MEP_OK;
  *(volatile int*)c->err_host = 0;
  static const char* msgs[] = {
      "ok",
      "timed out waiting for a peer's routing counts",
      "timed out waiting for a peer's dispatched rows",
      "timed out waiting for a peer's expert outputs",
      "a routing index is outside [0, num_experts)",
      "a receive buffer would overflow (raise recv_capacity_rows)",
      "an entry was routed to a rank that does not hold its expert",
      "debug wait timed out",
      "a tensor-core pipeline barrier timed out",
      "timed out waiting for a peer at a rank barrier",
  };
  const int nmsg = (int)(sizeof(msgs) / sizeof(msgs[0]));
  return fail(c, MEP_ERR_DEVICE,
              std::string("device error: ") + (code > 0 && code < nmsg ? msgs[code] : "unknown"));
}

int mep_set_option(mep_ctx* c, const char* name, int64_t value) {
  if (!c || !name) return MEP_ERR_INVALID;
  if (!std::strcmp(name, "force_simt")) {
    c->force_simt = value != 0;
    return MEP_OK;
  }
  if (!std::strcmp(name, "tc_single_cta")) {
    c->tc_single_cta = value != 0;
    return MEP_OK;
  }
  if (!std::strcmp(name, "ffn_ast")) {
    c->ffn_ast = value != 0;
    return MEP_OK;
  }
  if (!std::strcmp(name, "ffn_prefetch")) {
    c->ffn_prefetch = value != 0;
    return MEP_OK;
  }
  if (!std::strcmp(name, "router_no_tc")) {
    c->router_no_tc = value != 0;
    return MEP_OK;
  }
  if (!std::strcmp(name, "dispatch_per_warp")) {
    c->dispatch_per_warp = value != 0;
    return MEP_OK;
  }
  if (!std::strcmp(name, "timeline")) {
    c->tl_on = value != 0;
    return MEP_OK;
  }
  if (!std::strcmp(name, "timeout_ms")) {
    if (value < 1) return fail(c, MEP_ERR_INVALID, "timeout_ms must be >= 1");
    c->timeout_ns = (unsigned long long)value * 1000000ull;
    return MEP_OK;
  }
  return fail(c, MEP_ERR_INVALID, std::string("unknown option ") + name);
}

int mep_barrier(mep_ctx* c, void* stream) {
  if (!c) return MEP_ERR_INVALID;
  if (int rc = check_peers(c)) return rc;
  if (int rc = use_device(c)) return rc;
  launch_rank_barrier(c->peers, c->world, c->rank, c->seq + 1,
                      reinterpret_cast<const uint32_t*>(c->sym + c->off_flags), wait_cfg(c),
                      tl_of(c), as_stream(stream));
  MEP_CK(c, cudaGetLastError());
  return MEP_OK;
}

int mep_read_timeline(mep_ctx* c, uint64_t* out, void* stream) {
  if (!c || !out) return fail(c, MEP_ERR_INVALID, "NULL argument");
  if (int rc = use_device(c)) return rc;
  cudaStream_t st = as_stream(stream);
  MEP_CK(c, cudaMemcpyAsync(out, c->tl, (size_t)kTlSlots * sizeof(uint64_t),
                            cudaMemcpyDeviceToHost, st));
  MEP_CK(c, cudaStreamSynchronize(st));
  MEP_CK(c, cudaMemsetAsync(c->tl, 0, (size_t)kTlSlots * sizeof(uint64_t), st));
  return MEP_OK;
}

int mep_debug_wait(mep_ctx* c, uint32_t target, int64_t timeout_ms, void* stream) {
  if (!c) return MEP_ERR_INVALID;
  if (timeout_ms < 1) return fail(c, MEP_ERR_INVALID, "timeout_ms must be >= 1");
  if (int rc = use_device(c)) return rc;
  WaitCfg wc{c->err_dev, (unsigned long long)timeout_ms * 1000000ull};
  launch_wait_flags(reinterpret_cast<const uint32_t*>(c->sym + c->off_flags), 0, 1, nullptr,
                    target, kErrWaitDebug, wc, nullptr, 0, as_stream(stream));
  MEP_CK(c, cudaGetLastError());
  return MEP_OK;
}

}  // extern "C"
