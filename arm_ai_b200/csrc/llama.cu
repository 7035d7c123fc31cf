// llama.cu — quantized-Llama model: GGUF load, decode step (PDL + CUDA graph),
// prefill, greedy generate. C ABI in include/armai.h.
#include <math.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "decode_mega.cuh"
#include "gguf.h"
#include "gemm_tc.cuh"
#include "fa_tc.cuh"
#include "nccl_dyn.h"
#include "llama_kernels.cuh"

using namespace armai;

namespace {

constexpr int PREFILL_TILE = 8;       // tokens per prefill matvec launch
constexpr int BATCH_NB = 16;          // sequences per batched-decode matvec launch
constexpr int BATCH_NB_WIDE = 8;      // ... when 16 activation rows of K do not fit shared memory
constexpr int TC_PREFILL_MIN = 64;    // prompts this long use the tensor-core GEMM (prefill_gemm 0)

constexpr int ATTN_TOK_PER_LAUNCH = 64;
constexpr uint32_t STAGE_MAX = 44 * 1024;
constexpr size_t SMEM_LIMIT = 227 * 1024;   // hard per-CTA limit
constexpr size_t SMEM_DECODE = 110 * 1024;  // decode kernels: two CTAs per SM for PDL overlap

struct DevMat {
  uint8_t* w = nullptr;
  int type = 0;
  int rows = 0, cols = 0;
  int row_bytes = 0;
  Seg seg() const { return Seg{w, type, rows, cols / QK_K, row_bytes}; }
};

struct Layer {
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  DevMat wq, wk, wv, wo, wg, wu, wd;
};

struct Plan {
  int grid = 0, rows_per_cta = 0, chunk_rows = 0, ns = 0;
  uint32_t stage_bytes = 0;
  size_t smem = 0;
};

}  // namespace

struct armai_llama {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  bool broken = false;
  // hyper-parameters
  int n_layer = 0, n_embd = 0, n_ff = 0, n_head = 0, n_head_kv = 0, head_dim = 0, rope_dim = 0;
  int n_vocab = 0, max_seq = 4096, max_batch = 1, kv_f16 = 0;
  float eps = 1e-5f, rope_base = 10000.f;
  bool use_graph = true, use_pdl = true;
  // weights
  uint8_t* arena = nullptr;
  size_t arena_bytes = 0;
  std::vector<Layer> layers;
  DevMat tok_embd, output;
  float* out_norm = nullptr;
  int64_t weight_bytes_per_token = 0;
  // tables and caches
  float* cos_t = nullptr;
  float* sin_t = nullptr;
  void* kc = nullptr;
  void* vc = nullptr;
  int64_t kv_seq_stride = 0, kv_layer_stride = 0;
  // decode activations (max_batch rows)
  float *x = nullptr, *q = nullptr, *y = nullptr, *h = nullptr, *logits = nullptr;
  uint32_t* d_token = nullptr;
  int* d_pos = nullptr;
  uint32_t* d_err = nullptr;
  float* attn_part = nullptr;
  unsigned* attn_cnt = nullptr;
  size_t attn_cap_tokens = 0;
  float* am_val = nullptr;
  int* am_idx = nullptr;
  unsigned* am_cnt = nullptr;
  // prefill buffers
  int pf_cap = 0;
  float *pX = nullptr, *pQ = nullptr, *pY = nullptr, *pH = nullptr;
  int* p_pos = nullptr;
  uint32_t* p_tok = nullptr;
  uint8_t* pA = nullptr;       // tensor-core GEMM A tiles
  float* pG = nullptr;         // GEMM output [cap][g_cols]
  int g_cols = 0;
  float* pWs = nullptr;        // GEMM split-K partials
  size_t ws_floats = 0;
  uint8_t *pFq = nullptr, *pFk = nullptr, *pFv = nullptr;  // prompt attention operand tiles
  int prefill_gemm = 0;        // armai_llama_opts.prefill_gemm
  int batch_gemm = 0;          // armai_llama_opts.batch_gemm
  bool q80 = false;            // a matrix takes Q8_0 activations (Q4_0 / Q5_0 / Q8_0)
  // tensor parallelism (tp > 1): this rank holds a slice of every matrix, the
  // residual stream x is replicated, row-split products are summed by NCCL
  int tp = 1, tp_rank = 0;
  void* comm = nullptr;
  int v0 = 0, v_stride = 0;      // first vocab row of this rank; vocab rows per rank
  float* tp_part = nullptr;      // [max_batch][E] partial sums of a row-split matvec
  float* best_val = nullptr;     // [max_batch] head winner: value and local row
  int* best_idx = nullptr;
  uint32_t* tp_send = nullptr;   // [max_batch][2]: winner bits, global row
  uint32_t* tp_recv = nullptr;   // [tp][max_batch][2]
  float* logits_all = nullptr;   // [tp * v_stride] gathered logits
  void* xchg = nullptr;          // persistent kernel: this rank's exchange area (IPC-shared)
  void* peer_xchg[8] = {};       // the other ranks' exchange areas, mapped here
  void* flow = nullptr;          // persistent kernel: tagged words (q, K/V row, y, h, row sums) + epoch
  // pinned host staging
  uint32_t* h_tok = nullptr;   // ring of 8 token slots
  int* h_misc = nullptr;       // small pinned scratch
  uint32_t* h_prompt = nullptr;
  size_t h_prompt_cap = 0;
  // plans
  Plan pl_qkv1, pl_wo1, pl_gu1, pl_down1, pl_head1;
  Plan pl_qkvT, pl_woT, pl_guT, pl_downT;
  Plan pl_qkvB, pl_woB, pl_guB, pl_downB, pl_headB;  // batched decode (max_batch > 1)
  int batch_nb = 16;             // sequences per batched matvec launch (BATCH_NB or BATCH_NB_WIDE)
  uint32_t* h_btok = nullptr;  // pinned [max_batch] tokens of a batched step
  size_t attn_smem = 0;
  int n_kernels_step = 0;
  cudaGraphExec_t graph = nullptr;
  cudaGraphExec_t bgraph = nullptr;  // batched GEMM step for bgraph_n sequences
  int bgraph_n = 0;
  int kv_len = 0;  // positions currently in the cache (host mirror)
  size_t device_bytes = 0;
  // persistent decode kernel
  bool use_mega = true;
  MkPhase* d_phases = nullptr;
  MkParams mk;
  size_t mk_smem = 0;
  int mk_grid = 0;
};

namespace {

// Activations a launch's rows need (candle's VecDotType): bit 1 Q8_K for
// k-quant rows, bit 2 Q8_0 for legacy-type rows.
int seg_acts(const Seg* seg, int nseg) {
  int a = 0;
  for (int i = 0; i < nseg; i++) a |= is_legacy(seg[i].type) ? 2 : 1;
  return a;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Row plan for a k_matvec launch: contiguous row ranges per CTA, chunks that
// fit a stage, a ring of up to 3 stages within the shared-memory budget.
Plan make_plan(int total_rows, int unit, int row_bytes_per_unit_row, int rows_per_unit_in_stage,
               int K, int NB, bool norm, int nsm, size_t budget, bool q80) {
  Plan p;
  // rows of the virtual row space per CTA, rounded up to `unit`
  int per = (total_rows + nsm - 1) / nsm;
  per = ((per + unit - 1) / unit) * unit;
  p.rows_per_cta = per;
  p.grid = (total_rows + per - 1) / per;
  const size_t act = mv_smem_layout(0, 0, K, NB, norm, q80).total;
  const size_t unit_bytes = (size_t)row_bytes_per_unit_row * rows_per_unit_in_stage;  // bytes per row of the chunk
  const size_t room = budget > act + 1024 ? budget - act - 1024 : 0;
  size_t stage_cap = std::min<size_t>(STAGE_MAX, room);
  int chunk = (int)(stage_cap / unit_bytes);
  chunk = (chunk / unit) * unit;
  if (chunk < unit) chunk = unit;
  if (chunk > per) chunk = per;
  p.chunk_rows = chunk;
  p.stage_bytes = (uint32_t)al16((size_t)chunk * unit_bytes);
  const int nchunks = (per + chunk - 1) / chunk;
  int ns = std::min(nchunks, 3);
  while (ns > 1 && act + (size_t)ns * p.stage_bytes + 1024 > budget) ns--;
  p.ns = ns;
  p.smem = mv_smem_layout(ns, p.stage_bytes, K, NB, norm, q80).total;
  return p;
}

template <int MODE, int NB>
int set_smem_attr(size_t smem) {
  ARMAI_CUDA(cudaFuncSetAttribute(k_matvec<MODE, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
  return ARMAI_OK;
}

template <int MODE, int NB>
cudaError_t launch_mv(armai_llama* m, const Plan& pl, MvParams p, int nrows = NB) {
  p.nrows = nrows;
  return launch_k(k_matvec<MODE, NB>, dim3(pl.grid), dim3(MV_THREADS), pl.smem, m->stream,
                  m->use_pdl, p);
}

MvParams base_params(armai_llama* m, const Plan& pl) {
  MvParams p;
  std::memset(&p, 0, sizeof p);
  p.eps = m->eps;
  p.rows_per_cta = pl.rows_per_cta;
  p.chunk_rows = pl.chunk_rows;
  p.ns = pl.ns;
  p.stage_bytes = pl.stage_bytes;
  p.err = m->d_err;
  p.hd = m->head_dim;
  p.max_seq = m->max_seq;
  p.kv_f16 = m->kv_f16;
  p.cos_t = m->cos_t;
  p.sin_t = m->sin_t;
  return p;
}

void* kv_layer_ptr(armai_llama* m, void* base, int l) {
  const size_t es = m->kv_f16 ? 2 : 4;
  return (uint8_t*)base + (size_t)l * m->kv_layer_stride * es;
}

// KV cache of sequence slot `seq` in layer l.
void* kv_seq_ptr(armai_llama* m, void* base, int l, int seq) {
  const size_t es = m->kv_f16 ? 2 : 4;
  return (uint8_t*)kv_layer_ptr(m, base, l) + (size_t)seq * m->kv_seq_stride * es;
}

// ---- one layer's launches for NB tokens whose activations live at x/q/y/h ----
template <int NB>
cudaError_t launch_qkv(armai_llama* m, const Plan& pl, int l, const float* x, float* q,
                       const int* pos, int64_t kv_seq_stride, int seq = 0, int nrows = NB) {
  const Layer& L = m->layers[l];
  MvParams p = base_params(m, pl);
  p.x = x;
  p.gamma = L.attn_norm;
  p.K = m->n_embd;
  p.nb = m->n_embd / QK_K;
  p.seg[0] = L.wq.seg();
  p.seg[1] = L.wk.seg();
  p.seg[2] = L.wv.seg();
  p.nseg = 3;
  p.acts = seg_acts(p.seg, p.nseg);
  p.qn = L.wq.rows;
  p.kn = L.wk.rows;
  p.total_rows = L.wq.rows + L.wk.rows + L.wv.rows;
  p.out = q;
  p.out_stride = m->n_head * m->head_dim;
  p.kc = kv_seq_ptr(m, m->kc, l, seq);
  p.vc = kv_seq_ptr(m, m->vc, l, seq);
  p.kv_seq_stride = kv_seq_stride;
  p.pos = pos;
  return launch_mv<MODE_QKV, NB>(m, pl, p, nrows);
}

template <int NB>
cudaError_t launch_resid(armai_llama* m, const Plan& pl, const DevMat& w, const float* in,
                         float* x, int nrows = NB) {
  MvParams p = base_params(m, pl);
  p.x = in;
  p.gamma = nullptr;
  p.K = w.cols;
  p.nb = w.cols / QK_K;
  p.seg[0] = w.seg();
  p.nseg = 1;
  p.acts = seg_acts(p.seg, p.nseg);
  p.total_rows = w.rows;
  p.out = x;
  p.out_stride = m->n_embd;
  return launch_mv<MODE_RESID, NB>(m, pl, p, nrows);
}

template <int NB>
cudaError_t launch_gateup(armai_llama* m, const Plan& pl, int l, const float* x, float* h,
                          int nrows = NB) {
  const Layer& L = m->layers[l];
  MvParams p = base_params(m, pl);
  p.x = x;
  p.gamma = L.ffn_norm;
  p.K = m->n_embd;
  p.nb = m->n_embd / QK_K;
  p.seg[0] = L.wg.seg();
  p.seg[1] = L.wu.seg();
  p.nseg = 2;
  p.acts = seg_acts(p.seg, p.nseg);
  p.total_rows = L.wg.rows;
  p.out = h;
  p.out_stride = m->n_ff;
  return launch_mv<MODE_GATEUP, NB>(m, pl, p, nrows);
}

// Output norm + logits + argmax for `nrows` rows of x (plan pl_head1 for one
// row, pl_headB for a batch): token[b] = argmax, pos_out[b] = pos[b] + 1.
template <int NB>
cudaError_t launch_head(armai_llama* m, const Plan& pl, const float* x, const int* pos, int* pos_out,
                        uint32_t* token, int nrows = NB, int best_off = 0) {
  MvParams p = base_params(m, pl);
  p.x = x;
  p.gamma = m->out_norm;
  p.K = m->n_embd;
  p.nb = m->n_embd / QK_K;
  p.seg[0] = m->output.seg();
  p.nseg = 1;
  p.acts = seg_acts(p.seg, p.nseg);
  p.total_rows = m->output.rows;
  p.out = m->logits;
  p.out_stride = m->n_vocab;
  p.am_val = m->am_val;
  p.am_idx = m->am_idx;
  p.counter = m->am_cnt;
  p.token = token;
  p.pos = pos;
  p.pos_out = pos_out;
  if (m->tp > 1) {
    p.best_val = m->best_val + best_off;
    p.best_idx = m->best_idx + best_off;
  }
  return launch_mv<MODE_HEAD, NB>(m, pl, p, nrows);
}

cudaError_t launch_attn(armai_llama* m, int l, const float* q, float* y, const int* pos, int nb_tok,
                        int64_t kv_seq_stride, int seq = 0) {
  AttnParams a;
  a.q = q;
  a.kc = kv_seq_ptr(m, m->kc, l, seq);
  a.vc = kv_seq_ptr(m, m->vc, l, seq);
  a.kv_seq_stride = kv_seq_stride;
  a.kv_f16 = m->kv_f16;
  a.pos = pos;
  a.max_seq = m->max_seq;
  a.hd = m->head_dim;
  a.n_head = m->n_head;
  a.n_kv = m->n_head_kv;
  a.scale = (float)(1.0 / sqrt((double)m->head_dim));
  a.part = m->attn_part;
  a.counters = m->attn_cnt;
  a.y = y;
  a.err = m->d_err;
  const dim3 grid(m->n_head_kv, ATT_SPLITS, nb_tok), block(ATT_THREADS);
  if (m->head_dim == 64)
    return m->kv_f16 ? launch_k(k_attn_decode<64, __half>, grid, block, m->attn_smem, m->stream, m->use_pdl, a)
                     : launch_k(k_attn_decode<64, float>, grid, block, m->attn_smem, m->stream, m->use_pdl, a);
  return m->kv_f16 ? launch_k(k_attn_decode<128, __half>, grid, block, m->attn_smem, m->stream, m->use_pdl, a)
                   : launch_k(k_attn_decode<128, float>, grid, block, m->attn_smem, m->stream, m->use_pdl, a);
}

cudaError_t launch_embed(armai_llama* m, const uint32_t* tokens, float* x, int n) {
  return launch_k(k_embed, dim3(n), dim3(256), 0, m->stream, m->use_pdl,
                  (const uint8_t*)m->tok_embd.w, m->tok_embd.type, m->n_embd / QK_K,
                  (int64_t)m->tok_embd.row_bytes, tokens, x, m->n_embd, m->n_vocab, m->d_err);
}

cudaError_t launch_mega(armai_llama* m) {
  // the grid-barrier counter starts at 0: set at setup, reset by the kernel's
  // last CTA at the end of every step
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m->mk_grid);
  cfg.blockDim = dim3(MK_THREADS);
  cfg.dynamicSmemBytes = m->mk_smem;
  cfg.stream = m->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (m->head_dim == 64)
    return m->kv_f16 ? cudaLaunchKernelEx(&cfg, k_decode_mega<64, __half>, m->mk)
                     : cudaLaunchKernelEx(&cfg, k_decode_mega<64, float>, m->mk);
  return m->kv_f16 ? cudaLaunchKernelEx(&cfg, k_decode_mega<128, __half>, m->mk)
                   : cudaLaunchKernelEx(&cfg, k_decode_mega<128, float>, m->mk);
}

// Tensor parallelism in the persistent kernel: each rank's exchange area
// (head counter at 128, head winners at 256, generation-tagged residual slots
// at XCHG_SLOTS_OFF) is shared with the other ranks through CUDA IPC; the
// handles travel by one NCCL all-gather.
constexpr size_t XCHG_SLOTS_OFF = 512;
int wait_done(armai_llama* m, cudaEvent_t ev = nullptr);
int setup_peer_exchange(armai_llama* m, MkParams& k) {
  if (m->tp > MK_TP_MAX) return fail(ARMAI_E_INVALID, "tensor parallel: at most 8 ranks");
  const size_t E = m->n_embd;
  const size_t bytes = XCHG_SLOTS_OFF + 2 * (size_t)m->tp * E * 8;  // (generation, value) pairs
  ARMAI_CUDA(cudaMalloc(&m->xchg, bytes));
  ARMAI_CUDA(cudaMemset(m->xchg, 0, bytes));
  // Per rank: its IPC handle (64 B) and its GPU's UUID (16 B), all-gathered.
  struct Rec {
    cudaIpcMemHandle_t h;
    cudaUUID_t uuid;
  };
  static_assert(sizeof(cudaIpcMemHandle_t) == 64 && sizeof(Rec) == 80, "exchange record");
  Rec mine;
  ARMAI_CUDA(cudaIpcGetMemHandle(&mine.h, m->xchg));
  cudaDeviceProp prop;
  ARMAI_CUDA(cudaGetDeviceProperties(&prop, m->device));
  mine.uuid = prop.uuid;
  void* dh = nullptr;
  ARMAI_CUDA(cudaMalloc(&dh, (size_t)m->tp * sizeof(Rec)));
  std::vector<Rec> all(m->tp);
  int rc = ARMAI_OK;
  cudaError_t e = cudaMemcpyAsync((uint8_t*)dh + (size_t)m->tp_rank * sizeof(Rec), &mine, sizeof(Rec),
                                  cudaMemcpyHostToDevice, m->stream);
  if (e == cudaSuccess)
    rc = nccl_allgather_b32((uint8_t*)dh + (size_t)m->tp_rank * sizeof(Rec), dh, sizeof(Rec) / 4, m->comm,
                            m->stream);
  if (e == cudaSuccess && rc == ARMAI_OK)
    e = cudaMemcpyAsync(all.data(), dh, (size_t)m->tp * sizeof(Rec), cudaMemcpyDeviceToHost, m->stream);
  if (e == cudaSuccess && rc == ARMAI_OK) rc = wait_done(m);
  cudaFree(dh);
  if (rc != ARMAI_OK) return rc;
  if (e != cudaSuccess) return cuda_fail(e, "exchange of IPC handles", __FILE__, __LINE__);
  // The ranks' persistent kernels wait on one another: they must run on
  // distinct GPUs (on one GPU nothing makes them resident at the same time).
  for (int a = 0; a < m->tp; a++)
    for (int b = a + 1; b < m->tp; b++)
      if (std::memcmp(&all[a].uuid, &all[b].uuid, sizeof(cudaUUID_t)) == 0)
        return fail(ARMAI_E_INVALID, "tensor parallel: ranks " + std::to_string(a) + " and " + std::to_string(b) +
                                         " are on the same GPU");
  for (int r = 0; r < m->tp; r++) {
    uint8_t* base = nullptr;
    if (r == m->tp_rank) {
      base = (uint8_t*)m->xchg;
    } else {
      void* pr = nullptr;
      ARMAI_CUDA(cudaIpcOpenMemHandle(&pr, all[r].h, cudaIpcMemLazyEnablePeerAccess));
      m->peer_xchg[r] = pr;
      base = (uint8_t*)pr;
    }
    k.hctr[r] = reinterpret_cast<unsigned long long*>(base + 128);
    k.hslot[r] = reinterpret_cast<uint32_t*>(base + 256);
    k.xslot[r] = reinterpret_cast<unsigned long long*>(base + XCHG_SLOTS_OFF);
  }
  return ARMAI_OK;
}

// Phase list and shared-memory layout of the persistent decode kernel.
int setup_mega(armai_llama* m, int nsm) {
  const int E = m->n_embd, F = m->n_ff, QN = m->n_head * m->head_dim;
  // Grid: one CTA per SM, but no more CTAs than the smallest matvec phase
  // has units (QKV: row pairs), so every CTA owns rows in every phase.
  int grid = nsm;
  for (const Layer& L : m->layers)
    grid = std::min({grid, (L.wq.rows + L.wk.rows + L.wv.rows) / 2, L.wo.rows, L.wg.rows, L.wd.rows});
  grid = std::min(grid, m->output.rows);
  if (grid < 1) return fail(ARMAI_E_INVALID, "persistent decode kernel: empty phase");
  // largest row count of a CTA (the balanced split gives each CTA the floor
  // or the ceiling of units / grid)
  auto per_cta = [&](int total, int unit) {
    const int units = (total + unit - 1) / unit;
    return ((units + grid - 1) / grid) * unit;
  };
  auto chunk_for = [&](int unit_bytes, int unit, int per) {
    int c = (int)(MK_STAGE / (uint32_t)unit_bytes);
    c = (c / unit) * unit;
    if (c < unit) c = unit;
    return std::min(c, per);
  };
  std::vector<MkPhase> ph;
  auto mat_phase = [&](int kind, int layer, std::initializer_list<const DevMat*> mats, int total, int unit,
                       int unit_bytes, int K, const float* gamma, float* out) {
    MkPhase p;
    std::memset(&p, 0, sizeof p);
    p.kind = kind;
    p.layer = layer;
    int i = 0;
    for (const DevMat* d : mats) p.seg[i++] = d->seg();
    p.nseg = i;
    p.acts = seg_acts(p.seg, p.nseg);
    p.total_rows = total;
    p.rows_per_cta = per_cta(total, unit);
    p.chunk_rows = chunk_for(unit_bytes, unit, p.rows_per_cta);
    p.K = K;
    p.nb = K / QK_K;
    p.gamma = gamma;
    p.out = out;
    if (layer >= 0) {
      p.kc = kv_layer_ptr(m, m->kc, layer);
      p.vc = kv_layer_ptr(m, m->vc, layer);
    }
    ph.push_back(p);
  };
  for (int l = 0; l < m->n_layer; l++) {
    const Layer& L = m->layers[l];
    const int qkv_rb = std::max(L.wq.row_bytes, std::max(L.wk.row_bytes, L.wv.row_bytes));
    mat_phase(PH_QKV, l, {&L.wq, &L.wk, &L.wv}, L.wq.rows + L.wk.rows + L.wv.rows, 2, qkv_rb, E, L.attn_norm,
              nullptr);
    MkPhase a;
    std::memset(&a, 0, sizeof a);
    a.kind = PH_ATTN;
    a.layer = l;
    a.kc = kv_layer_ptr(m, m->kc, l);
    a.vc = kv_layer_ptr(m, m->vc, l);
    ph.push_back(a);
    mat_phase(PH_WO, l, {&L.wo}, L.wo.rows, 1, L.wo.row_bytes, QN, nullptr, nullptr);
    mat_phase(PH_GATEUP, l, {&L.wg, &L.wu}, L.wg.rows, 1, L.wg.row_bytes + L.wu.row_bytes, E, L.ffn_norm, nullptr);
    mat_phase(PH_DOWN, l, {&L.wd}, L.wd.rows, 1, L.wd.row_bytes, F, nullptr, nullptr);
  }
  mat_phase(PH_HEAD, -1, {&m->output}, m->output.rows, 1, m->output.row_bytes, E, m->out_norm, m->logits);
  ARMAI_CUDA(cudaMalloc(&m->d_phases, ph.size() * sizeof(MkPhase)));
  ARMAI_CUDA(cudaMemcpy(m->d_phases, ph.data(), ph.size() * sizeof(MkPhase), cudaMemcpyHostToDevice));
  const int kmax = std::max(E, std::max(F, QN));
  MkParams& k = m->mk;
  std::memset(&k, 0, sizeof k);
  size_t o = 0;
  const int nrep = m->n_head / m->n_head_kv;
  // the attention region also holds the staged rmsnorm weights (n_embd f32)
  const size_t att_bytes = std::max(mk_att_floats(m->head_dim, nrep) * 4, (size_t)m->n_embd * 4) + 64;
  // Q8_0 activation buffers only when a matrix takes them (legacy types)
  const size_t act0 = m->q80 ? al16((size_t)kmax) + 2 * al16((size_t)kmax / QK8_0 * 4) : 0;
  size_t fixed = al16((size_t)(2 * MK_MAX_NS + 1) * 8) + al16((size_t)kmax) + al16((size_t)kmax / QK_K * 4) +
                 al16((size_t)kmax / 16 * 4) + al16((64 + (size_t)kmax / QK_K + 8) * 4) + al16(att_bytes) +
                 al16((size_t)E * 4) + act0;
  // 2 KB of headroom for the kernel's static shared memory (phase copies etc.)
  int ns = (int)std::min<size_t>(MK_MAX_NS, (SMEM_LIMIT - fixed - 2048) / MK_STAGE);
  if (ns < 2) return fail(ARMAI_E_INVALID, "persistent decode kernel: not enough shared memory");
  k.ns = ns;
  o = (size_t)ns * MK_STAGE;
  k.off_bars = o;   o += al16((size_t)(2 * MK_MAX_NS + 1) * 8);
  k.off_act_qs = o; o += al16((size_t)kmax);
  k.off_act_d = o;  o += al16((size_t)kmax / QK_K * 4);
  k.off_act_bs = o; o += al16((size_t)kmax / 16 * 4);
  k.off_red = o;    o += al16((64 + (size_t)kmax / QK_K + 8) * 4);
  k.off_att = o;    o += al16(att_bytes);
  k.off_xrep = o;   o += al16((size_t)E * 4);
  if (m->q80) {
    k.off_act0_qs = o; o += al16((size_t)kmax);
    k.off_act0_d = o;  o += al16((size_t)kmax / QK8_0 * 4);
    k.off_act0_s = o;  o += al16((size_t)kmax / QK8_0 * 4);
  }
  m->mk_smem = o;
  k.kmax = kmax;
  // Tagged words, zeroed (tag 0 is never awaited): q, the K/V row, y, h,
  // then (one rank) the row-sum slots, and the epoch.
  const size_t KVW = 2 * (size_t)m->n_head_kv * m->head_dim;
  const size_t nwords = 2 * (size_t)QN + KVW + F + (m->tp > 1 ? 0 : 2 * (size_t)E);
  ARMAI_CUDA(cudaMalloc(&m->flow, nwords * 8 + 64));
  ARMAI_CUDA(cudaMemset(m->flow, 0, nwords * 8 + 64));
  unsigned long long* fw = reinterpret_cast<unsigned long long*>(m->flow);
  k.fq = fw;
  k.fkv = fw + QN;
  k.fy = fw + QN + KVW;
  k.fh = fw + 2 * (size_t)QN + KVW;
  k.epoch = fw + nwords;
  k.tp = m->tp;
  k.tp_rank = m->tp_rank;
  k.v0 = m->v0;
  if (m->tp > 1) ARMAI_TRY(setup_peer_exchange(m, k));
  else k.xslot[0] = fw + 2 * (size_t)QN + KVW + F;
  k.ph = m->d_phases;
  k.n_ph = (int)ph.size();
  k.embd = m->tok_embd.w;
  k.embd_type = m->tok_embd.type;
  k.embd_row_bytes = m->tok_embd.row_bytes;
  k.n_embd = E;
  k.cos_t = m->cos_t;
  k.sin_t = m->sin_t;
  k.hd = m->head_dim;
  k.n_head = m->n_head;
  k.n_kv = m->n_head_kv;
  k.max_seq = m->max_seq;
  k.kv_f16 = m->kv_f16;
  k.eps = m->eps;
  k.att_scale = (float)(1.0 / sqrt((double)m->head_dim));
  k.att_part = m->attn_part;
  k.att_cnt = m->attn_cnt;
  k.am_val = m->am_val;
  k.am_idx = m->am_idx;
  k.am_cnt = m->am_cnt;
  k.token = m->d_token;
  k.pos = m->d_pos;
  k.err = m->d_err;
  k.poll_limit = MK_BAR_LIMIT;
  k.test_stall_phase = -1;
  m->mk_grid = grid;
  if (m->head_dim == 64) {
    ARMAI_CUDA(cudaFuncSetAttribute(k_decode_mega<64, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)o));
    ARMAI_CUDA(cudaFuncSetAttribute(k_decode_mega<64, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)o));
  } else {
    ARMAI_CUDA(cudaFuncSetAttribute(k_decode_mega<128, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)o));
    ARMAI_CUDA(cudaFuncSetAttribute(k_decode_mega<128, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)o));
  }
  // every CTA must be resident at once (CTAs wait for one another's outputs)
  int per_sm = 0;
  if (m->head_dim == 64)
    ARMAI_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_mega<64, float>, MK_THREADS, o));
  else
    ARMAI_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_mega<128, float>, MK_THREADS, o));
  if (per_sm < 1) return fail(ARMAI_E_INVALID, "persistent decode kernel does not fit one SM");
  return ARMAI_OK;
}

// The single-sequence decode step: token d_token at position d_pos.
// Tensor parallelism, winner of the head across ranks: (value, global row)
// of every rank, then the reference's argmax order (larger value, then the
// smaller row; NaN never wins).
// For n sequences: send[2s], send[2s + 1] = sequence s's winner on this rank;
// recv = every rank's send ([rank][n][2]).
__global__ void k_tp_pack(const float* best_val, const int* best_idx, int v0, uint32_t* send, int n) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= n) return;
  const int bi = best_idx[s];
  send[2 * s] = __float_as_uint(best_val[s]);
  send[2 * s + 1] = bi == 0x7fffffff ? 0xffffffffu : (uint32_t)(bi + v0);
}
__global__ void k_tp_pick(const uint32_t* recv, int tp, int n, uint32_t* token) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= n) return;
  float bv = -INFINITY;
  uint32_t bi = 0xffffffffu;
  for (int r = 0; r < tp; r++) {
    const float v = __uint_as_float(recv[((size_t)r * n + s) * 2]);
    const uint32_t i = recv[((size_t)r * n + s) * 2 + 1];
    if (i != 0xffffffffu && (bi == 0xffffffffu || v > bv || (v == bv && i < bi))) { bv = v; bi = i; }
  }
  token[s] = bi == 0xffffffffu ? 0u : bi;
}

int tp_head_merge(armai_llama* m, uint32_t* token, int n = 1) {
  const unsigned blocks = (unsigned)((n + 127) / 128);
  k_tp_pack<<<blocks, 128, 0, m->stream>>>(m->best_val, m->best_idx, m->v0, m->tp_send, n);
  ARMAI_CUDA(cudaGetLastError());
  ARMAI_TRY(nccl_allgather_b32(m->tp_send, m->tp_recv, (size_t)2 * n, m->comm, m->stream));
  k_tp_pick<<<blocks, 128, 0, m->stream>>>(m->tp_recv, m->tp, n, token);
  ARMAI_CUDA(cudaGetLastError());
  return ARMAI_OK;
}

// x += W y for a matrix split along K over the ranks: rank 0 adds its part
// into x, the others write theirs to tp_part, and an all-reduce sums them
// into x everywhere.
int rowsplit_resid(armai_llama* m, const Plan& pl, const DevMat& w, const float* y) {
  if (m->tp == 1) {
    ARMAI_CUDA(launch_resid<1>(m, pl, w, y, m->x));
    return ARMAI_OK;
  }
  if (m->tp_rank == 0) {
    ARMAI_CUDA(launch_resid<1>(m, pl, w, y, m->x));
  } else {
    MvParams p = base_params(m, pl);
    p.x = y;
    p.K = w.cols;
    p.nb = w.cols / QK_K;
    p.seg[0] = w.seg();
    p.nseg = 1;
    p.acts = seg_acts(p.seg, p.nseg);
    p.total_rows = w.rows;
    p.out = m->tp_part;
    p.out_stride = m->n_embd;
    const cudaError_t e = launch_mv<MODE_STORE, 1>(m, pl, p);
    ARMAI_CUDA(e);
  }
  return nccl_allreduce_sum_f32(m->tp_rank == 0 ? m->x : m->tp_part, m->x, (size_t)m->n_embd, m->comm, m->stream);
}

int enqueue_decode_step(armai_llama* m) {
  if (m->use_mega) {
    ARMAI_CUDA(launch_mega(m));
    return ARMAI_OK;
  }
  ARMAI_CUDA(launch_embed(m, m->d_token, m->x, 1));
  for (int l = 0; l < m->n_layer; l++) {
    ARMAI_CUDA(launch_qkv<1>(m, m->pl_qkv1, l, m->x, m->q, m->d_pos, 0));
    ARMAI_CUDA(launch_attn(m, l, m->q, m->y, m->d_pos, 1, 0));
    ARMAI_TRY(rowsplit_resid(m, m->pl_wo1, m->layers[l].wo, m->y));
    ARMAI_CUDA(launch_gateup<1>(m, m->pl_gu1, l, m->x, m->h));
    ARMAI_TRY(rowsplit_resid(m, m->pl_down1, m->layers[l].wd, m->h));
  }
  ARMAI_CUDA(launch_head<1>(m, m->pl_head1, m->x, m->d_pos, m->d_pos, m->d_token));
  if (m->tp > 1) ARMAI_TRY(tp_head_merge(m, m->d_token));
  return ARMAI_OK;
}

int run_decode_step(armai_llama* m) {
  if (m->graph) {
    ARMAI_CUDA(cudaGraphLaunch(m->graph, m->stream));
    return ARMAI_OK;
  }
  return enqueue_decode_step(m);
}

// Host wait on the model's stream (ev == nullptr) or on an event recorded on
// it. Tensor parallelism: a rank whose peer failed outside a collective would
// wait inside NCCL for ever, so the wait is bounded; on expiry the
// communicator is aborted (its kernels return), the model is marked broken and
// the call fails. One GPU: a plain synchronize.
constexpr double TP_WAIT_S = 120.0;
int wait_done(armai_llama* m, cudaEvent_t ev) {
  if (m->tp <= 1 || !m->comm) {
    ARMAI_CUDA(ev ? cudaEventSynchronize(ev) : cudaStreamSynchronize(m->stream));
    return ARMAI_OK;
  }
  const auto t0 = std::chrono::steady_clock::now();
  for (uint32_t it = 0;; ++it) {
    const cudaError_t e = ev ? cudaEventQuery(ev) : cudaStreamQuery(m->stream);
    if (e != cudaErrorNotReady) {
      ARMAI_CUDA(e);
      return ARMAI_OK;
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > TP_WAIT_S) {
      nccl_comm_abort(m->comm);
      m->comm = nullptr;
      m->broken = true;
      cudaStreamSynchronize(m->stream);
      return fail(ARMAI_E_DEVICE, "tensor parallel: no progress for " + std::to_string((int)TP_WAIT_S) +
                                      " s (another rank failed?); communicator aborted, reload the model");
    }
    if (it > 2000) std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

int check_device_error(armai_llama* m) {
  ARMAI_TRY(wait_done(m));
  ARMAI_CUDA(cudaMemcpy(m->h_misc, m->d_err, 4, cudaMemcpyDeviceToHost));
  if (m->h_misc[0] != 0) {
    m->broken = true;
    return fail(ARMAI_E_DEVICE, "device error flag 0x" + std::to_string(m->h_misc[0]) +
                                    " (bounded wait expired or bad token id); reload the model");
  }
  return ARMAI_OK;
}

int ensure_prefill(armai_llama* m, int S) {
  if (S <= m->pf_cap) return ARMAI_OK;
  if (m->bgraph) {  // it holds the buffers about to be replaced
    cudaGraphExecDestroy(m->bgraph);
    m->bgraph = nullptr;
    m->bgraph_n = 0;
  }
  int cap = std::max(S, 64);
  cap = ((cap + PREFILL_TILE - 1) / PREFILL_TILE) * PREFILL_TILE;
  cudaFree(m->pX); cudaFree(m->pQ); cudaFree(m->pY); cudaFree(m->pH);
  cudaFree(m->p_pos); cudaFree(m->p_tok); cudaFree(m->pA); cudaFree(m->pG); cudaFree(m->pWs);
  cudaFree(m->pFq); cudaFree(m->pFk); cudaFree(m->pFv);
  m->pX = m->pQ = m->pY = m->pH = m->pG = m->pWs = nullptr;
  m->pFq = m->pFk = m->pFv = nullptr;
  m->pA = nullptr;
  m->pf_cap = 0;
  m->ws_floats = 0;
  const size_t qn = (size_t)m->n_head * m->head_dim;
  if (m->prefill_gemm != 1 || m->batch_gemm != 1) {
    const Layer& L0 = m->layers[0];
    const int kmax = std::max(m->n_embd, std::max(m->n_ff, (int)qn));
    m->g_cols = std::max(L0.wq.rows + L0.wk.rows + L0.wv.rows, std::max(2 * m->n_ff, m->n_embd));
    ARMAI_CUDA(cudaMalloc(&m->pA, qgemm_a_bytes(cap, kmax)));
    ARMAI_CUDA(cudaMalloc(&m->pG, (size_t)cap * m->g_cols * 4));
    // split-K partials: a few splits of long prompts, many of short ones
    m->ws_floats = (size_t)m->g_cols * (size_t)std::max(2 * cap, 2048);
    ARMAI_CUDA(cudaMalloc(&m->pWs, m->ws_floats * 4));
    if (m->head_dim == 64 || m->head_dim == 128) {
      // attention operand tiles; zeroed once so that the key rows past a
      // prompt's end hold finite values (P = 0 there multiplies them)
      const size_t tiles = (size_t)(cap + 127) / 128, tb = fa_tile_bytes(m->head_dim);
      ARMAI_CUDA(cudaMalloc(&m->pFq, (size_t)m->n_head * tiles * tb));
      ARMAI_CUDA(cudaMalloc(&m->pFk, (size_t)m->n_head_kv * tiles * tb));
      ARMAI_CUDA(cudaMalloc(&m->pFv, (size_t)m->n_head_kv * tiles * tb));
      ARMAI_CUDA(cudaMemset(m->pFq, 0, (size_t)m->n_head * tiles * tb));
      ARMAI_CUDA(cudaMemset(m->pFk, 0, (size_t)m->n_head_kv * tiles * tb));
      ARMAI_CUDA(cudaMemset(m->pFv, 0, (size_t)m->n_head_kv * tiles * tb));
    }
  }
  ARMAI_CUDA(cudaMalloc(&m->pX, (size_t)cap * m->n_embd * 4));
  ARMAI_CUDA(cudaMalloc(&m->pQ, (size_t)cap * qn * 4));
  ARMAI_CUDA(cudaMalloc(&m->pY, (size_t)cap * qn * 4));
  ARMAI_CUDA(cudaMalloc(&m->pH, (size_t)cap * m->n_ff * 4));
  ARMAI_CUDA(cudaMalloc(&m->p_pos, (size_t)cap * 4));
  ARMAI_CUDA(cudaMalloc(&m->p_tok, (size_t)cap * 4));
  if ((size_t)cap > m->h_prompt_cap) {
    if (m->h_prompt) cudaFreeHost(m->h_prompt);
    m->h_prompt = nullptr;
    ARMAI_CUDA(cudaMallocHost(&m->h_prompt, (size_t)cap * 2 * 4));
    m->h_prompt_cap = cap;
  }
  m->pf_cap = cap;
  return ARMAI_OK;
}

// One weight GEMM of the tensor-core path over the activation tiles in pA.
int gemm_job(armai_llama* m, std::initializer_list<const DevMat*> mats, int S, int K, int mode, float* dst,
             int ldd, QgSplit* split = nullptr) {
  QgJob j;
  std::memset(&j, 0, sizeof j);
  j.a_tiles = m->pA;
  j.m = S;
  j.k = K;
  for (const DevMat* d : mats) j.seg[j.nseg++] = QgSeg{d->w, d->type, d->rows, d->row_bytes};
  j.mode = mode;
  j.dst = dst;
  j.ldd = ldd;
  j.ws = m->pWs;
  j.ws_floats = m->ws_floats;
  j.err = m->d_err;
  j.pdl = m->use_pdl;
  return qgemm_run(j, m->stream, split);
}

// One layer of S tokens through the tensor-core GEMMs. On entry pA holds the
// activation tiles of x normalised with L.attn_norm; on return x[S][E] has
// the layer's two residual adds and pA the tiles of the new x normalised with
// next_gamma (none when next_gamma is null). q/y are scratch rows. Token t
// sits at position pos[t] of sequence slot seq + t * seq_step (a prompt: one
// slot; a decode batch: slot t).
int gemm_layer(armai_llama* m, const Layer& L, int l, int S, float* x, float* q, float* y, const int* pos,
               int seq_step, int seq, const float* next_gamma) {
  const int E = m->n_embd, QN = m->n_head * m->head_dim, F = m->n_ff;
  const bool pdl = m->use_pdl;
  QgSplit g;
  ARMAI_TRY(gemm_job(m, {&L.wq, &L.wk, &L.wv}, S, E, QG_PARTIAL, nullptr, 0, &g));
  // a prompt (positions 0 .. S-1) with a tensor-core head dim: q / k / v also
  // as the attention kernel's operand tiles
  const bool fa = !seq_step && m->pFq;
  const int ntl = (S + 127) / 128;
  const FaTilesOut tl{m->pFq, m->pFk, m->pFv, ntl, ntl, (int)fa_tile_bytes(m->head_dim)};
  ARMAI_TRY(qkv_post_launch(g, S, pos, L.wq.rows, L.wk.rows, m->head_dim, m->max_seq, m->cos_t, m->sin_t,
                            fa ? nullptr : q, kv_seq_ptr(m, m->kc, l, seq), kv_seq_ptr(m, m->vc, l, seq),
                            m->kv_f16, m->kv_seq_stride, seq_step, m->stream, pdl, fa ? &tl : nullptr));
  if (seq_step) {
    ARMAI_CUDA(launch_attn(m, l, q, y, pos, S, m->kv_seq_stride, seq));
  } else if (fa) {
    // the prompt's causal attention on the tensor cores (positions 0 .. S-1)
    FaParams a{};
    a.qt = m->pFq;
    a.kt = m->pFk;
    a.vt = m->pFv;
    a.nqt = a.nkt = ntl;
    a.o = y;
    a.o_ts = QN;
    a.o_hs = m->head_dim;
    a.sq = a.sk = S;
    a.n_head = m->n_head;
    a.group = m->n_head / m->n_head_kv;
    a.scale = (float)(1.0 / sqrt((double)m->head_dim));
    a.causal = 1;
    a.err = m->d_err;
    ARMAI_TRY(fa_tc_launch(a, m->head_dim, 1, m->stream, pdl));
  } else {
    for (int t0 = 0; t0 < S; t0 += ATTN_TOK_PER_LAUNCH) {
      const int n = std::min(ATTN_TOK_PER_LAUNCH, S - t0);
      ARMAI_CUDA(launch_attn(m, l, q + (size_t)t0 * QN, y + (size_t)t0 * QN, pos + t0, n, 0, seq));
    }
  }
  // x += W in (attn_output / ffn_down), then the next activation tiles;
  // tensor parallel: the ranks' partial products are summed by NCCL first
  auto resid = [&](const DevMat& w, int K, const float* gamma) -> int {
    QgSplit r;
    if (m->tp == 1) {
      ARMAI_TRY(gemm_job(m, {&w}, S, K, QG_PARTIAL, nullptr, 0, &r));
    } else {
      ARMAI_TRY(gemm_job(m, {&w}, S, K, QG_STORE, m->pG, E));
      ARMAI_TRY(nccl_allreduce_sum_f32(m->pG, m->pG, (size_t)S * E, m->comm, m->stream));
      r = QgSplit{m->pG, 1, 0, E};
    }
    return resid_act_launch(r, x, S, E, gamma, m->eps, gamma ? m->pA : nullptr, m->stream, pdl);
  };
  ARMAI_TRY(qgemm_act_launch(y, nullptr, m->eps, S, QN, m->pA, m->stream, pdl));
  ARMAI_TRY(resid(L.wo, QN, L.ffn_norm));
  ARMAI_TRY(gemm_job(m, {&L.wg, &L.wu}, S, E, QG_PARTIAL, nullptr, 0, &g));
  ARMAI_TRY(silu_act_launch(g, S, F, m->pA, m->stream, pdl));
  ARMAI_TRY(resid(L.wd, F, next_gamma));
  return ARMAI_OK;
}

// Prefill of S >= 2 tokens at positions 0..S-1 (index_pos 0: fresh cache).
// Integer path: the same Q8_K x Q4_K/Q6_K kernels as decode, over tiles of
// PREFILL_TILE tokens (weights streamed once per tile), and the split-K
// attention with per-token causal limits.
// Prompt of S tokens at positions 0..S-1 into sequence slot `seq` (its KV
// cache); the head writes the first generated token to d_token[seq] and S to
// d_pos[seq].
int enqueue_prefill(armai_llama* m, const uint32_t* tokens, int S, int seq = 0) {
  ARMAI_TRY(ensure_prefill(m, S));
  uint32_t* ht = m->h_prompt;
  int* hp = reinterpret_cast<int*>(m->h_prompt + m->h_prompt_cap);
  // The pinned staging may still be read by an earlier async copy.
  ARMAI_TRY(wait_done(m));
  for (int i = 0; i < S; i++) { ht[i] = tokens[i]; hp[i] = i; }
  ARMAI_CUDA(cudaMemcpyAsync(m->p_tok, ht, (size_t)S * 4, cudaMemcpyHostToDevice, m->stream));
  ARMAI_CUDA(cudaMemcpyAsync(m->p_pos, hp, (size_t)S * 4, cudaMemcpyHostToDevice, m->stream));
  const size_t E = m->n_embd, QN = (size_t)m->n_head * m->head_dim, F = m->n_ff;
  ARMAI_CUDA(launch_embed(m, m->p_tok, m->pX, S));
  const bool gemm = m->prefill_gemm == 2 || (m->prefill_gemm == 0 && S >= TC_PREFILL_MIN);
  if (gemm)
    ARMAI_TRY(qgemm_act_launch(m->pX, m->layers[0].attn_norm, m->eps, S, (int)E, m->pA, m->stream, m->use_pdl));
  for (int l = 0; l < m->n_layer && gemm; l++) {
    const float* next = l + 1 < m->n_layer ? m->layers[l + 1].attn_norm : nullptr;
    ARMAI_TRY(gemm_layer(m, m->layers[l], l, S, m->pX, m->pQ, m->pY, m->p_pos, 0, seq, next));
  }
  for (int l = 0; l < m->n_layer && !gemm; l++) {
    int t = 0;
    for (; t + PREFILL_TILE <= S; t += PREFILL_TILE)
      ARMAI_CUDA(launch_qkv<PREFILL_TILE>(m, m->pl_qkvT, l, m->pX + t * E, m->pQ + t * QN, m->p_pos + t, 0, seq));
    for (; t < S; t++)
      ARMAI_CUDA(launch_qkv<1>(m, m->pl_qkv1, l, m->pX + t * E, m->pQ + t * QN, m->p_pos + t, 0, seq));
    for (int t0 = 0; t0 < S; t0 += ATTN_TOK_PER_LAUNCH) {
      const int n = std::min(ATTN_TOK_PER_LAUNCH, S - t0);
      ARMAI_CUDA(launch_attn(m, l, m->pQ + t0 * QN, m->pY + t0 * QN, m->p_pos + t0, n, 0, seq));
    }
    t = 0;
    for (; t + PREFILL_TILE <= S; t += PREFILL_TILE)
      ARMAI_CUDA(launch_resid<PREFILL_TILE>(m, m->pl_woT, m->layers[l].wo, m->pY + t * QN, m->pX + t * E));
    for (; t < S; t++)
      ARMAI_CUDA(launch_resid<1>(m, m->pl_wo1, m->layers[l].wo, m->pY + t * QN, m->pX + t * E));
    t = 0;
    for (; t + PREFILL_TILE <= S; t += PREFILL_TILE)
      ARMAI_CUDA(launch_gateup<PREFILL_TILE>(m, m->pl_guT, l, m->pX + t * E, m->pH + t * F));
    for (; t < S; t++)
      ARMAI_CUDA(launch_gateup<1>(m, m->pl_gu1, l, m->pX + t * E, m->pH + t * F));
    t = 0;
    for (; t + PREFILL_TILE <= S; t += PREFILL_TILE)
      ARMAI_CUDA(launch_resid<PREFILL_TILE>(m, m->pl_downT, m->layers[l].wd, m->pH + t * F, m->pX + t * E));
    for (; t < S; t++)
      ARMAI_CUDA(launch_resid<1>(m, m->pl_down1, m->layers[l].wd, m->pH + t * F, m->pX + t * E));
  }
  ARMAI_CUDA(launch_head<1>(m, m->pl_head1, m->pX + (size_t)(S - 1) * E, m->p_pos + (S - 1), m->d_pos + seq,
                            m->d_token + seq));
  if (m->tp > 1) ARMAI_TRY(tp_head_merge(m, m->d_token + seq));
  return ARMAI_OK;
}

// One greedy decode step for sequence slots 0..n-1: token d_token[b] at
// position d_pos[b] of slot b's KV cache; writes the next token and position
// back. Matvecs run BATCH_NB sequences per weight pass.
// x[s] += W in[s] for the n sequences of a batched step (W = attn_output or
// ffn_down, in = y or h with row stride W.cols). Tensor parallel: W is split
// along K; rank 0 adds its part into x, the others store theirs in tp_part,
// and one all-reduce of n rows sums them into x everywhere.
template <int NB>
int rowsplit_resid_batch(armai_llama* m, const Plan& pl, const DevMat& w, const float* in, int n) {
  const size_t E = m->n_embd, K = (size_t)w.cols;
  for (int g = 0; g < n; g += NB) {
    const int nr = std::min(NB, n - g);
    if (m->tp == 1 || m->tp_rank == 0) {
      ARMAI_CUDA(launch_resid<NB>(m, pl, w, in + g * K, m->x + g * E, nr));
    } else {
      MvParams p = base_params(m, pl);
      p.x = in + g * K;
      p.K = w.cols;
      p.nb = w.cols / QK_K;
      p.seg[0] = w.seg();
      p.nseg = 1;
      p.acts = seg_acts(p.seg, p.nseg);
      p.total_rows = w.rows;
      p.out = m->tp_part + g * E;
      p.out_stride = m->n_embd;
      const cudaError_t e = launch_mv<MODE_STORE, NB>(m, pl, p, nr);
      ARMAI_CUDA(e);
    }
  }
  if (m->tp == 1) return ARMAI_OK;
  return nccl_allreduce_sum_f32(m->tp_rank == 0 ? m->x : m->tp_part, m->x, (size_t)n * E, m->comm, m->stream);
}

template <int NB>
int enqueue_batch_step_nb(armai_llama* m, int n) {
  const size_t E = m->n_embd, QN = (size_t)m->n_head * m->head_dim, F = m->n_ff;
  ARMAI_CUDA(launch_embed(m, m->d_token, m->x, n));
  for (int l = 0; l < m->n_layer; l++) {
    const Layer& L = m->layers[l];
    for (int g = 0; g < n; g += NB)
      ARMAI_CUDA(launch_qkv<NB>(m, m->pl_qkvB, l, m->x + g * E, m->q + g * QN, m->d_pos + g, m->kv_seq_stride,
                                g, std::min(NB, n - g)));
    ARMAI_CUDA(launch_attn(m, l, m->q, m->y, m->d_pos, n, m->kv_seq_stride, 0));
    ARMAI_TRY(rowsplit_resid_batch<NB>(m, m->pl_woB, L.wo, m->y, n));
    for (int g = 0; g < n; g += NB)
      ARMAI_CUDA(launch_gateup<NB>(m, m->pl_guB, l, m->x + g * E, m->h + g * F, std::min(NB, n - g)));
    ARMAI_TRY(rowsplit_resid_batch<NB>(m, m->pl_downB, L.wd, m->h, n));
  }
  for (int g = 0; g < n; g += NB)
    ARMAI_CUDA(launch_head<NB>(m, m->pl_headB, m->x + g * E, m->d_pos + g, m->d_pos + g, m->d_token + g,
                               std::min(NB, n - g), g));
  if (m->tp > 1) ARMAI_TRY(tp_head_merge(m, m->d_token, n));
  return ARMAI_OK;
}

// The batched step through the tensor-core GEMMs (one GPU, Q4_K / Q6_K):
// per layer one GEMM per weight group for all n sequences, attention per
// sequence slot, then the logits GEMM (its activation tiles carry the output
// norm) and a row argmax.
int enqueue_batch_step_gemm(armai_llama* m, int n) {
  ARMAI_TRY(ensure_prefill(m, std::max(n, 64)));
  const int E = m->n_embd;
  ARMAI_CUDA(launch_embed(m, m->d_token, m->x, n));
  ARMAI_TRY(qgemm_act_launch(m->x, m->layers[0].attn_norm, m->eps, n, E, m->pA, m->stream, m->use_pdl));
  for (int l = 0; l < m->n_layer; l++) {
    const float* next = l + 1 < m->n_layer ? m->layers[l + 1].attn_norm : m->out_norm;
    ARMAI_TRY(gemm_layer(m, m->layers[l], l, n, m->x, m->q, m->y, m->d_pos, 1, 0, next));
  }
  ARMAI_TRY(gemm_job(m, {&m->output}, n, E, QG_STORE, m->logits, m->n_vocab));
  if (m->tp == 1) return row_argmax_launch(m->logits, n, m->output.rows, m->n_vocab, m->d_token, m->d_pos, m->stream,
                                           m->use_pdl);
  // tensor parallel: this rank's vocab rows; the ranks' winners are merged
  ARMAI_TRY(row_argmax_launch(m->logits, n, m->output.rows, m->n_vocab, m->d_token, m->d_pos, m->stream, m->use_pdl,
                              m->best_val, m->best_idx));
  return tp_head_merge(m, m->d_token, n);
}

int enqueue_batch_step(armai_llama* m, int n) {
  if (m->batch_gemm != 1) {
    if (!m->use_graph) return enqueue_batch_step_gemm(m, n);
    // one graph per batch size, captured on first use (its buffers are
    // allocated first; a later reallocation drops the graph)
    ARMAI_TRY(ensure_prefill(m, std::max(n, 64)));
    if (m->bgraph_n != n) {
      if (m->bgraph) cudaGraphExecDestroy(m->bgraph);
      m->bgraph = nullptr;
      m->bgraph_n = 0;
      cudaGraph_t gr = nullptr;
      ARMAI_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
      const int erc = enqueue_batch_step_gemm(m, n);
      const cudaError_t ec = cudaStreamEndCapture(m->stream, &gr);
      if (erc != ARMAI_OK || ec != cudaSuccess) {
        if (gr) cudaGraphDestroy(gr);
        return erc != ARMAI_OK ? erc : cuda_fail(ec, "cudaStreamEndCapture", __FILE__, __LINE__);
      }
      const cudaError_t ce = cudaGraphInstantiate(&m->bgraph, gr, 0);
      cudaGraphDestroy(gr);
      if (ce != cudaSuccess) return cuda_fail(ce, "cudaGraphInstantiate", __FILE__, __LINE__);
      m->bgraph_n = n;
    }
    ARMAI_CUDA(cudaGraphLaunch(m->bgraph, m->stream));
    return ARMAI_OK;
  }
  return m->batch_nb == BATCH_NB ? enqueue_batch_step_nb<BATCH_NB>(m, n)
                                 : enqueue_batch_step_nb<BATCH_NB_WIDE>(m, n);
}

// Single token at position `pos` through the decode kernels.
int enqueue_single(armai_llama* m, uint32_t token, int pos) {
  ARMAI_TRY(wait_done(m));
  m->h_misc[1] = (int)token;
  m->h_misc[2] = pos;
  ARMAI_CUDA(cudaMemcpyAsync(m->d_token, &m->h_misc[1], 4, cudaMemcpyHostToDevice, m->stream));
  ARMAI_CUDA(cudaMemcpyAsync(m->d_pos, &m->h_misc[2], 4, cudaMemcpyHostToDevice, m->stream));
  return run_decode_step(m);
}

// forward(tokens, index_pos) semantics shared by armai_llama_forward and generate.
int forward_locked(armai_llama* m, const uint32_t* tokens, int n, int index_pos) {
  if (n <= 0) return fail(ARMAI_E_INVALID, "forward: empty input");
  for (int i = 0; i < n; i++)
    if (tokens[i] >= (uint32_t)m->n_vocab)
      return fail(ARMAI_E_INVALID, "forward: token id " + std::to_string(tokens[i]) +
                                       " out of range for vocab " + std::to_string(m->n_vocab));
  if ((int64_t)index_pos + n > m->max_seq)
    return fail(ARMAI_E_RANGE, "forward: positions " + std::to_string(index_pos) + ".." +
                                   std::to_string(index_pos + n - 1) +
                                   " exceed the rotary table (max_seq_len " +
                                   std::to_string(m->max_seq) + ")");
  if (index_pos == 0) m->kv_len = 0;
  if (index_pos != m->kv_len)
    return fail(ARMAI_E_INVALID, "forward: index_pos " + std::to_string(index_pos) +
                                     " does not continue the cache (length " +
                                     std::to_string(m->kv_len) + ")");
  if (n > 1 && index_pos != 0)
    return fail(ARMAI_E_INVALID,
                "forward: a multi-token step after the prompt is not supported (the causal mask "
                "covers only index_pos 0)");
  if (n == 1) ARMAI_TRY(enqueue_single(m, tokens[0], index_pos));
  else ARMAI_TRY(enqueue_prefill(m, tokens, n));
  m->kv_len = index_pos + n;
  return ARMAI_OK;
}

// ---------------------------------------------------------------------------
// Loading.
// ---------------------------------------------------------------------------
bool md_u32(const GgufFile& g, const std::string& key, int64_t& out) {
  auto it = g.kv.find(key);
  if (it == g.kv.end()) return false;
  if (it->second.kind != GgufValue::UINT && it->second.kind != GgufValue::INT) return false;
  out = it->second.i;
  return true;
}
bool md_f32(const GgufFile& g, const std::string& key, double& out) {
  auto it = g.kv.find(key);
  if (it == g.kv.end()) return false;
  if (it->second.kind == GgufValue::ARRAY || it->second.kind == GgufValue::STRING) return false;
  out = it->second.f;
  return true;
}

struct TensorJob {
  const GgufTensor* t;
  DevMat* mat;      // for matrices
  float** vec;      // for f32 vectors (norms)
  int64_t r0 = 0, nr = -1;   // row slice (tensor parallelism)
  int64_t b0 = 0, nbk = -1;  // super-block slice along K (tensor parallelism)
};

int upload_tensors(armai_llama* m, const char* path, const GgufFile& g, std::vector<TensorJob>& jobs) {
  FILE* f = fopen(path, "rb");
  if (!f) return fail(ARMAI_E_IO, std::string("open ") + path + " failed");
  const size_t STG = 64ull << 20;
  uint8_t* stg[2] = {nullptr, nullptr};
  uint8_t* rep = nullptr;
  cudaEvent_t ev[2];
  int rc = ARMAI_OK;
  if (cudaMallocHost(&stg[0], STG) != cudaSuccess || cudaMallocHost(&stg[1], STG) != cudaSuccess) {
    fclose(f);
    if (stg[0]) cudaFreeHost(stg[0]);
    return fail(ARMAI_E_NOMEM, "pinned staging allocation failed");
  }
  rep = (uint8_t*)malloc(STG);
  cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming);
  cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming);
  cudaEventRecord(ev[0], m->stream);
  cudaEventRecord(ev[1], m->stream);
  int slot = 0;
  for (TensorJob& j : jobs) {
    const GgufTensor& t = *j.t;
    const int64_t rows = j.nr >= 0 ? j.nr : t.rows(), full_cols = t.cols();
    const int64_t full_rb = ggml_row_bytes(t.type, full_cols);
    const bool kslice = j.mat && j.nbk >= 0;
    const int64_t cols = kslice ? j.nbk * QK_K : full_cols;
    const int64_t raw_rb = ggml_row_bytes(t.type, cols);
    const int64_t boff = kslice ? ggml_row_bytes(t.type, j.b0 * QK_K) : 0;
    int64_t rows_per = std::max<int64_t>(1, (int64_t)(STG / (size_t)std::max<int64_t>(full_rb, 1)));
    if (j.mat && t.type == GGML_Q6_K) rows_per = std::max<int64_t>(1, (int64_t)(STG / (size_t)dev_row_bytes(GGML_Q6_K, full_cols)));
    if (fseeko(f, (off_t)(g.data_offset + t.offset + (uint64_t)j.r0 * full_rb), SEEK_SET) != 0) {
      rc = fail(ARMAI_E_IO, "seek failed");
      break;
    }
    uint8_t* dst = j.mat ? j.mat->w : (uint8_t*)*j.vec;
    for (int64_t r0 = 0; r0 < rows && rc == ARMAI_OK; r0 += rows_per) {
      const int64_t nr = std::min(rows_per, rows - r0);
      cudaEventSynchronize(ev[slot]);
      uint8_t* buf = stg[slot];
      const bool via_rep = (j.mat && t.type == GGML_Q6_K) || kslice;
      if (fread(via_rep ? rep : buf, 1, (size_t)(nr * full_rb), f) != (size_t)(nr * full_rb)) {
        rc = fail(ARMAI_E_IO, "short read of tensor '" + t.name + "'");
        break;
      }
      if (kslice)  // keep each row's super-blocks [b0, b0 + nbk)
        for (int64_t r = 0; r < nr; r++) memmove(rep + r * raw_rb, rep + r * full_rb + boff, (size_t)raw_rb);
      size_t out_bytes = (size_t)(nr * raw_rb);
      if (j.mat && t.type == GGML_Q6_K) {
        repack_q6k_rows(rep, nr, cols, buf);
        out_bytes = (size_t)(nr * dev_row_bytes(GGML_Q6_K, cols));
      } else if (kslice) {
        memcpy(buf, rep, out_bytes);
      } else if (!j.mat && t.type == GGML_F16) {
        // f16 vector -> f32 (candle dequantises norm weights at load)
        float* tmp = (float*)rep;
        const uint16_t* hsrc = (const uint16_t*)buf;
        for (int64_t i = 0; i < nr * cols; i++) {
          __half hv = __ushort_as_half(hsrc[i]);
          tmp[i] = __half2float(hv);
        }
        memcpy(buf, tmp, (size_t)(nr * cols * 4));
        out_bytes = (size_t)(nr * cols * 4);
      }
      const size_t drb = j.mat ? (size_t)j.mat->row_bytes : (size_t)cols * 4;
      if (cudaMemcpyAsync(dst + (size_t)r0 * drb, buf, out_bytes, cudaMemcpyHostToDevice, m->stream) != cudaSuccess) {
        rc = fail(ARMAI_E_CUDA, "upload of '" + t.name + "' failed");
        break;
      }
      cudaEventRecord(ev[slot], m->stream);
      slot ^= 1;
    }
    if (rc != ARMAI_OK) break;
  }
  cudaStreamSynchronize(m->stream);
  cudaEventDestroy(ev[0]);
  cudaEventDestroy(ev[1]);
  cudaFreeHost(stg[0]);
  cudaFreeHost(stg[1]);
  free(rep);
  fclose(f);
  return rc;
}

void free_model(armai_llama* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  if (m->stream) wait_done(m);
  if (m->graph) cudaGraphExecDestroy(m->graph);  // before the NCCL communicator it may hold
  if (m->bgraph) cudaGraphExecDestroy(m->bgraph);
  if (m->comm && m->xchg && !m->broken) {
    // no rank may still write into this rank's exchange area: meet first
    float* one = nullptr;
    if (cudaMalloc(&one, 4) == cudaSuccess) {
      nccl_allreduce_sum_f32(one, one, 1, m->comm, m->stream);
      wait_done(m);
      cudaFree(one);
    }
  }
  for (void* pp : m->peer_xchg)
    if (pp) cudaIpcCloseMemHandle(pp);
  if (m->comm) nccl_comm_destroy(m->comm);
  void* dptrs[] = {m->arena, m->cos_t, m->sin_t, m->kc, m->vc, m->x, m->q, m->y, m->h, m->logits,
                   m->d_token, m->d_pos, m->d_err, m->attn_part, m->attn_cnt, m->am_val, m->am_idx,
                   m->am_cnt, m->pX, m->pQ, m->pY, m->pH, m->p_pos, m->p_tok, m->d_phases, m->flow,
                   m->pA, m->pG, m->pWs, m->tp_part, m->best_val, m->best_idx, m->tp_send, m->tp_recv,
                   m->logits_all, m->xchg};
  for (void* p : dptrs)
    if (p) cudaFree(p);
  for (Layer& L : m->layers) { (void)L; }
  if (m->h_tok) cudaFreeHost(m->h_tok);
  if (m->h_btok) cudaFreeHost(m->h_btok);
  if (m->h_misc) cudaFreeHost(m->h_misc);
  if (m->h_prompt) cudaFreeHost(m->h_prompt);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

int load_model(const char* path, const armai_llama_opts* opts, armai_llama** out) {
  GgufFile g;
  ARMAI_TRY(gguf_read(path, g));
  auto it = g.kv.find("general.architecture");
  if (it != g.kv.end() && it->second.kind == GgufValue::STRING && it->second.s != "llama")
    return fail(ARMAI_E_FORMAT, "ModelWeights::from_gguf failed: unsupported architecture '" + it->second.s + "' (llama.* keys required)");
  int64_t n_expert = 0;
  if (md_u32(g, "llama.expert_count", n_expert) && n_expert > 1)
    return fail(ARMAI_E_FORMAT, "ModelWeights::from_gguf failed: mixture-of-experts models are not supported");
  int64_t head_count, head_count_kv, block_count, embd, rope_dim;
  double eps, freq_base = 10000.0;
  const char* req[] = {"llama.attention.head_count", "llama.attention.head_count_kv", "llama.block_count",
                       "llama.embedding_length", "llama.rope.dimension_count"};
  int64_t* dst[] = {&head_count, &head_count_kv, &block_count, &embd, &rope_dim};
  for (int i = 0; i < 5; i++)
    if (!md_u32(g, req[i], *dst[i]))
      return fail(ARMAI_E_FORMAT, std::string("ModelWeights::from_gguf failed: cannot find ") + req[i] + " in metadata");
  if (!md_f32(g, "llama.attention.layer_norm_rms_epsilon", eps))
    return fail(ARMAI_E_FORMAT, "ModelWeights::from_gguf failed: cannot find llama.attention.layer_norm_rms_epsilon in metadata");
  md_f32(g, "llama.rope.freq_base", freq_base);

  auto* m = new armai_llama();
  armai_llama_opts o;
  armai_llama_default_opts(&o);
  if (opts) o = *opts;
  m->device = o.device;
  m->max_seq = o.max_seq_len > 0 ? o.max_seq_len : 4096;
  m->kv_f16 = o.kv_f16 ? 1 : 0;
  m->max_batch = std::max(1, o.max_batch);
  m->use_graph = o.use_graph != 0;
  m->use_pdl = o.use_pdl != 0;
  m->use_mega = o.decode_kernel == 0;
  m->prefill_gemm = o.prefill_gemm;
  if (o.prefill_gemm < 0 || o.prefill_gemm > 2) {
    delete m;
    return fail(ARMAI_E_INVALID, "prefill_gemm must be 0, 1 or 2");
  }
  m->batch_gemm = o.batch_gemm;
  if (o.batch_gemm < 0 || o.batch_gemm > 2) {
    delete m;
    return fail(ARMAI_E_INVALID, "batch_gemm must be 0, 1 or 2");
  }
  m->tp = std::max(1, o.tp_size);
  m->tp_rank = o.tp_rank;
  if (m->tp > 1) {
    if (o.tp_rank < 0 || o.tp_rank >= m->tp || !o.tp_unique_id) {
      delete m;
      return fail(ARMAI_E_INVALID, "tensor parallel: tp_rank must be in [0, tp_size) and tp_unique_id set");
    }
    if (o.prefill_gemm == 1) {
      delete m;
      return fail(ARMAI_E_INVALID, "tensor parallel: prompts run the GEMM path (prefill_gemm 1 is not "
                                   "available with tp_size > 1)");
    }
    // decode: the persistent kernel sums the row-split products through peer
    // memory (decode_kernel 0), or the per-kernel chain through NCCL (1)
    m->use_pdl = false;
    m->prefill_gemm = 2;
  }
  m->n_layer = (int)block_count;
  m->n_embd = (int)embd;
  m->n_head = (int)head_count;
  m->n_head_kv = (int)head_count_kv;
  m->head_dim = (int)(embd / head_count);
  m->rope_dim = (int)rope_dim;
  m->eps = (float)eps;
  m->rope_base = (float)freq_base;
  if (m->n_head <= 0 || m->n_head_kv <= 0 || m->n_head % m->n_head_kv || embd % head_count ||
      m->rope_dim != m->head_dim || m->head_dim % 2 || m->n_embd % QK_K) {
    delete m;
    return fail(ARMAI_E_FORMAT, "ModelWeights::from_gguf failed: unsupported head geometry");
  }
  if (m->n_head / m->n_head_kv > ATT_MAX_REP || (m->head_dim != 64 && m->head_dim != 128)) {
    delete m;
    return fail(ARMAI_E_FORMAT, "unsupported attention geometry (query heads per KV head > 8, or head_dim not 64 or 128)");
  }
  {
    // the persistent kernel's attention is specialised for 1, 2, 4 or 8
    // query heads per KV head; other groupings take the per-kernel chain
    const int nrep = m->n_head / m->n_head_kv;
    if (nrep & (nrep - 1)) m->use_mega = false;
  }

  auto find = [&](const std::string& name) -> const GgufTensor* {
    auto t = g.tensors.find(name);
    return t == g.tensors.end() ? nullptr : &t->second;
  };
  std::vector<TensorJob> jobs;
  size_t arena = 0;
  int rc = ARMAI_OK;
  auto add_mat = [&](const std::string& name, DevMat& dm, int64_t want_cols, int64_t want_rows, int64_t r0 = 0,
                     int64_t nr = -1, int64_t b0 = 0, int64_t nbk = -1) -> int {
    const GgufTensor* t = find(name);
    if (!t) return fail(ARMAI_E_FORMAT, "ModelWeights::from_gguf failed: cannot find tensor info for " + name);
    if (t->dims.size() != 2) return fail(ARMAI_E_FORMAT, "tensor " + name + " is not 2-D");
    if (!is_kquant((int)t->type) && !is_legacy((int)t->type))
      return fail(ARMAI_E_FORMAT, std::string("tensor ") + name + " has type " + ggml_type_name(t->type) +
                                      "; this build supports Q4_0, Q5_0, Q8_0, Q4_K, Q5_K and Q6_K matrices");
    if ((want_cols > 0 && t->cols() != want_cols) || (want_rows > 0 && t->rows() != want_rows))
      return fail(ARMAI_E_FORMAT, "tensor " + name + " has an unexpected shape");
    dm.type = (int)t->type;
    dm.rows = (int)(nr >= 0 ? nr : t->rows());
    dm.cols = (int)(nbk >= 0 ? nbk * QK_K : t->cols());
    dm.row_bytes = (int)dev_row_bytes(dm.type, dm.cols);
    dm.w = reinterpret_cast<uint8_t*>(arena);  // offset for now
    arena += al16((size_t)dm.row_bytes * dm.rows + 255) & ~size_t(255);
    m->weight_bytes_per_token += (int64_t)dm.row_bytes * dm.rows;
    TensorJob job{t, &dm, nullptr};
    job.r0 = r0;
    job.nr = nr;
    job.b0 = b0;
    job.nbk = nbk;
    jobs.push_back(job);
    return ARMAI_OK;
  };
  std::vector<float*> vec_offsets;
  auto add_vec = [&](const std::string& name, float*& dv, int64_t n) -> int {
    const GgufTensor* t = find(name);
    if (!t) return fail(ARMAI_E_FORMAT, "ModelWeights::from_gguf failed: cannot find tensor info for " + name);
    if (t->type != GGML_F32 && t->type != GGML_F16)
      return fail(ARMAI_E_FORMAT, "norm tensor " + name + " must be F32 or F16");
    if ((int64_t)(t->rows() * t->cols()) != n) return fail(ARMAI_E_FORMAT, "tensor " + name + " has an unexpected shape");
    dv = reinterpret_cast<float*>(arena);
    arena += (size_t)((n * 4 + 255) & ~int64_t(255));
    m->weight_bytes_per_token += n * 4;
    jobs.push_back(TensorJob{t, nullptr, &dv});
    return ARMAI_OK;
  };
  const GgufTensor* te = find("token_embd.weight");
  if (!te) { delete m; return fail(ARMAI_E_FORMAT, "ModelWeights::from_gguf failed: cannot find tensor info for token_embd.weight"); }
  m->n_vocab = (int)te->rows();
  m->layers.resize(m->n_layer);
  rc = add_mat("token_embd.weight", m->tok_embd, m->n_embd, -1);
  // token_embd streams one row per token, not the whole table
  if (rc == ARMAI_OK) m->weight_bytes_per_token -= (int64_t)m->tok_embd.row_bytes * (m->tok_embd.rows - 1);
  if (rc == ARMAI_OK) rc = add_vec("output_norm.weight", m->out_norm, m->n_embd);
  const int T = m->tp, TR = m->tp_rank;
  // tensor parallelism: vocab rows of the head split in contiguous blocks
  m->v_stride = (m->n_vocab + T - 1) / T;
  m->v0 = std::min(TR * m->v_stride, m->n_vocab);
  const int64_t v_rows = std::min(m->v_stride, m->n_vocab - m->v0);
  if (T > 1 && v_rows <= 0) rc = fail(ARMAI_E_INVALID, "tensor parallel: more ranks than vocab rows");
  if (rc == ARMAI_OK) {
    if (find("output.weight")) rc = add_mat("output.weight", m->output, m->n_embd, m->n_vocab, m->v0, T > 1 ? v_rows : -1);
    else if (T > 1) {
      rc = add_mat("token_embd.weight", m->output, m->n_embd, -1, m->v0, v_rows);  // tied, this rank's rows
    } else {
      m->output = m->tok_embd;  // tied: candle falls back to token_embd
      m->weight_bytes_per_token += (int64_t)m->output.row_bytes * (m->output.rows - 1);
    }
  }
  const int64_t QN = (int64_t)m->n_head * m->head_dim, KN = (int64_t)m->n_head_kv * m->head_dim;
  if (rc == ARMAI_OK && T > 1 &&
      (m->n_head % T || m->n_head_kv % T || (QN / T) % QK_K))
    rc = fail(ARMAI_E_INVALID, "tensor parallel: " + std::to_string(T) + " ranks must divide the query heads (" +
                                   std::to_string(m->n_head) + ") and KV heads (" + std::to_string(m->n_head_kv) +
                                   ") with whole 256-value blocks of attn_output per rank");
  const int64_t QNl = QN / T, KNl = KN / T;
  for (int l = 0; l < m->n_layer && rc == ARMAI_OK; l++) {
    Layer& L = m->layers[l];
    const std::string p = "blk." + std::to_string(l) + ".";
    const int64_t sl = T > 1 ? 1 : 0;  // slice only when sharded
    rc = add_mat(p + "attn_q.weight", L.wq, m->n_embd, QN, TR * QNl * sl, sl ? QNl : -1);
    if (!rc) rc = add_mat(p + "attn_k.weight", L.wk, m->n_embd, KN, TR * KNl * sl, sl ? KNl : -1);
    if (!rc) rc = add_mat(p + "attn_v.weight", L.wv, m->n_embd, KN, TR * KNl * sl, sl ? KNl : -1);
    if (!rc) rc = add_mat(p + "attn_output.weight", L.wo, QN, m->n_embd, 0, -1, TR * (QNl / QK_K) * sl,
                          sl ? QNl / QK_K : -1);
    int64_t F = 0;
    if (!rc) {
      const GgufTensor* tg = find(p + "ffn_gate.weight");
      F = tg && tg->dims.size() == 2 ? tg->rows() : 0;
      if (T > 1 && (F % ((int64_t)T * QK_K)))
        rc = fail(ARMAI_E_INVALID, "tensor parallel: feed-forward length " + std::to_string(F) +
                                       " does not split into whole 256-value blocks over " + std::to_string(T) + " ranks");
    }
    const int64_t Fl = T > 1 ? F / T : -1;
    if (!rc) rc = add_mat(p + "ffn_gate.weight", L.wg, m->n_embd, -1, T > 1 ? TR * Fl : 0, Fl);
    if (!rc) { m->n_ff = (int)F; rc = add_mat(p + "ffn_up.weight", L.wu, m->n_embd, m->n_ff, T > 1 ? TR * Fl : 0, Fl); }
    if (!rc) rc = add_mat(p + "ffn_down.weight", L.wd, m->n_ff, m->n_embd, 0, -1, T > 1 ? TR * (Fl / QK_K) : 0,
                          T > 1 ? Fl / QK_K : -1);
    if (!rc) rc = add_vec(p + "attn_norm.weight", L.attn_norm, m->n_embd);
    if (!rc) rc = add_vec(p + "ffn_norm.weight", L.ffn_norm, m->n_embd);
    if (!rc && (m->n_ff % QK_K)) rc = fail(ARMAI_E_FORMAT, "feed-forward length must be a multiple of 256");
  }
  if (rc != ARMAI_OK) { delete m; return rc; }
  // Matrices other than Q4_K / Q6_K (Q5_K, and the legacy Q4_0 / Q5_0 /
  // Q8_0 whose dot products take Q8_0 activations): their prompts run the
  // integer per-kernel chain, as candle computes them, not the tensor-core
  // GEMM (whose shared activation operand serves one activation type).
  {
    std::vector<const DevMat*> mats{&m->tok_embd};
    if (find("output.weight")) mats.push_back(&m->output);
    for (const Layer& L : m->layers)
      for (const DevMat* d : {&L.wq, &L.wk, &L.wv, &L.wo, &L.wg, &L.wu, &L.wd}) mats.push_back(d);
    const DevMat* other = nullptr;
    for (const DevMat* d : mats) {
      if (is_legacy(d->type)) m->q80 = true;
      if (d->type != GGML_Q4_K && d->type != GGML_Q6_K && !other) other = d;
    }
    if (other) {
      if (T > 1) {
        delete m;
        return fail(ARMAI_E_INVALID, std::string("tensor parallel needs Q4_K / Q6_K matrices (its prompts run the "
                                                 "tensor-core GEMM); this model has ") + ggml_type_name(other->type));
      }
      m->prefill_gemm = 1;
      m->batch_gemm = 1;
    }
  }
  if (T > 1) {  // from here on the model is this rank's shard
    m->n_head /= T;
    m->n_head_kv /= T;
    m->n_ff /= T;
  }

  cudaError_t ce = cudaSetDevice(m->device);
  if (ce != cudaSuccess) { delete m; return cuda_fail(ce, "cudaSetDevice", __FILE__, __LINE__); }
#define LOAD_CUDA(call)                                                   \
  do {                                                                    \
    cudaError_t _e = (call);                                              \
    if (_e != cudaSuccess) {                                              \
      int _r = cuda_fail(_e, #call, __FILE__, __LINE__);                  \
      free_model(m);                                                      \
      return _r;                                                          \
    }                                                                     \
  } while (0)
  LOAD_CUDA(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
  m->arena_bytes = arena;
  LOAD_CUDA(cudaMalloc(&m->arena, arena));
  // rebase arena offsets to device pointers
  auto rebase = [&](uint8_t*& p) { p = m->arena + reinterpret_cast<size_t>(p); };
  for (TensorJob& j : jobs) {
    if (j.mat) rebase(j.mat->w);
    else { uint8_t* q = reinterpret_cast<uint8_t*>(*j.vec); rebase(q); *j.vec = reinterpret_cast<float*>(q); }
  }
  if (!find("output.weight")) m->output = m->tok_embd;
  rc = upload_tensors(m, path, g, jobs);
  if (rc != ARMAI_OK) { free_model(m); return rc; }

  // rotary tables: precomput_freqs_cis of candle quantized_llama
  {
    const int half = m->rope_dim / 2;
    std::vector<float> theta(half), c((size_t)m->max_seq * half), s((size_t)m->max_seq * half);
    for (int i = 0; i < m->rope_dim; i += 2)
      theta[i / 2] = 1.0f / powf(m->rope_base, (float)i / (float)m->rope_dim);
    for (int p = 0; p < m->max_seq; p++)
      for (int j = 0; j < half; j++) {
        const float a = (float)p * theta[j];
        c[(size_t)p * half + j] = cosf(a);
        s[(size_t)p * half + j] = sinf(a);
      }
    LOAD_CUDA(cudaMalloc(&m->cos_t, c.size() * 4));
    LOAD_CUDA(cudaMalloc(&m->sin_t, s.size() * 4));
    LOAD_CUDA(cudaMemcpy(m->cos_t, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
    LOAD_CUDA(cudaMemcpy(m->sin_t, s.data(), s.size() * 4, cudaMemcpyHostToDevice));
  }
  // KV cache [layer][seq][kv_head][max_seq][head_dim]
  m->kv_seq_stride = (int64_t)m->n_head_kv * m->max_seq * m->head_dim;
  m->kv_layer_stride = m->kv_seq_stride * m->max_batch;
  const size_t kv_bytes = (size_t)m->kv_layer_stride * m->n_layer * (m->kv_f16 ? 2 : 4);
  LOAD_CUDA(cudaMalloc(&m->kc, kv_bytes));
  LOAD_CUDA(cudaMalloc(&m->vc, kv_bytes));
  LOAD_CUDA(cudaMemsetAsync(m->kc, 0, kv_bytes, m->stream));
  LOAD_CUDA(cudaMemsetAsync(m->vc, 0, kv_bytes, m->stream));
  const int B = m->max_batch;
  LOAD_CUDA(cudaMalloc(&m->x, (size_t)B * m->n_embd * 4));
  LOAD_CUDA(cudaMalloc(&m->q, (size_t)B * QN * 4));
  LOAD_CUDA(cudaMalloc(&m->y, (size_t)B * QN * 4));
  LOAD_CUDA(cudaMalloc(&m->h, (size_t)B * m->n_ff * 4));
  LOAD_CUDA(cudaMalloc(&m->logits, (size_t)B * m->n_vocab * 4));
  LOAD_CUDA(cudaMalloc(&m->d_token, (size_t)std::max(B, 8) * 4));
  LOAD_CUDA(cudaMalloc(&m->d_pos, (size_t)std::max(B, 8) * 4));
  LOAD_CUDA(cudaMalloc(&m->d_err, 64));
  LOAD_CUDA(cudaMemsetAsync(m->d_err, 0, 64, m->stream));
  LOAD_CUDA(cudaMemsetAsync(m->d_token, 0, (size_t)std::max(B, 8) * 4, m->stream));
  LOAD_CUDA(cudaMemsetAsync(m->d_pos, 0, (size_t)std::max(B, 8) * 4, m->stream));
  const int nrep = m->n_head / m->n_head_kv;
  m->attn_cap_tokens = (size_t)std::max(B, ATTN_TOK_PER_LAUNCH);
  LOAD_CUDA(cudaMalloc(&m->attn_part, m->attn_cap_tokens * m->n_head_kv * ATT_SPLITS * nrep * (m->head_dim + 2) * 4));
  LOAD_CUDA(cudaMalloc(&m->attn_cnt, m->attn_cap_tokens * m->n_head_kv * 4));
  LOAD_CUDA(cudaMemsetAsync(m->attn_cnt, 0, m->attn_cap_tokens * m->n_head_kv * 4, m->stream));
  const int nsm = sm_count();
  LOAD_CUDA(cudaMalloc(&m->am_val, (size_t)B * nsm * 4));
  LOAD_CUDA(cudaMalloc(&m->am_idx, (size_t)B * nsm * 4));
  LOAD_CUDA(cudaMalloc(&m->am_cnt, 64));
  LOAD_CUDA(cudaMemsetAsync(m->am_cnt, 0, 64, m->stream));
  if (m->tp > 1) {
    LOAD_CUDA(cudaMalloc(&m->tp_part, (size_t)B * m->n_embd * 4));
    LOAD_CUDA(cudaMalloc(&m->best_val, (size_t)B * 4));
    LOAD_CUDA(cudaMalloc(&m->best_idx, (size_t)B * 4));
    LOAD_CUDA(cudaMalloc(&m->tp_send, (size_t)B * 8));
    LOAD_CUDA(cudaMalloc(&m->tp_recv, (size_t)m->tp * B * 8));
    LOAD_CUDA(cudaMalloc(&m->logits_all, (size_t)m->tp * m->v_stride * 4));
    const int nrc = nccl_comm_init(&m->comm, m->tp, opts->tp_unique_id, m->tp_rank);
    if (nrc != ARMAI_OK) { free_model(m); return nrc; }
  }
  LOAD_CUDA(cudaMallocHost(&m->h_tok, 64));
  LOAD_CUDA(cudaMallocHost(&m->h_misc, 64));

  // launch plans
  auto maxrb = [](const DevMat& a, const DevMat& b, const DevMat& c) {
    return std::max(a.row_bytes, std::max(b.row_bytes, c.row_bytes));
  };
  const Layer& L0 = m->layers[0];
  int qkv_rb = 0, gu_rb = 0, wo_rb = 0, dn_rb = 0;
  for (const Layer& L : m->layers) {
    qkv_rb = std::max(qkv_rb, maxrb(L.wq, L.wk, L.wv));
    gu_rb = std::max(gu_rb, L.wg.row_bytes + L.wu.row_bytes);
    wo_rb = std::max(wo_rb, L.wo.row_bytes);
    dn_rb = std::max(dn_rb, L.wd.row_bytes);
  }
  const int qkv_rows = L0.wq.rows + L0.wk.rows + L0.wv.rows;
  m->pl_qkv1 = make_plan(qkv_rows, 2, qkv_rb, 1, m->n_embd, 1, true, nsm, SMEM_DECODE, m->q80);
  m->pl_wo1 = make_plan(m->n_embd, 1, wo_rb, 1, (int)QN, 1, false, nsm, SMEM_DECODE, m->q80);
  m->pl_gu1 = make_plan(m->n_ff, 1, gu_rb, 1, m->n_embd, 1, true, nsm, SMEM_DECODE, m->q80);
  m->pl_down1 = make_plan(m->n_embd, 1, dn_rb, 1, m->n_ff, 1, false, nsm, SMEM_DECODE, m->q80);
  m->pl_head1 = make_plan(m->output.rows, 1, m->output.row_bytes, 1, m->n_embd, 1, true, nsm, SMEM_DECODE, m->q80);
  m->pl_qkvT = make_plan(qkv_rows, 2, qkv_rb, 1, m->n_embd, PREFILL_TILE, true, nsm, SMEM_LIMIT, m->q80);
  m->pl_woT = make_plan(m->n_embd, 1, wo_rb, 1, (int)QN, PREFILL_TILE, false, nsm, SMEM_LIMIT, m->q80);
  m->pl_guT = make_plan(m->n_ff, 1, gu_rb, 1, m->n_embd, PREFILL_TILE, true, nsm, SMEM_LIMIT, m->q80);
  m->pl_downT = make_plan(m->n_embd, 1, dn_rb, 1, m->n_ff, PREFILL_TILE, false, nsm, SMEM_LIMIT, m->q80);
  for (const Plan* pl : {&m->pl_qkv1, &m->pl_wo1, &m->pl_gu1, &m->pl_down1, &m->pl_head1, &m->pl_qkvT,
                         &m->pl_woT, &m->pl_guT, &m->pl_downT})
    if (pl->smem > SMEM_LIMIT) { free_model(m); return fail(ARMAI_E_INVALID, "model rows too wide for shared memory"); }
  int arc = set_smem_attr<MODE_QKV, 1>(m->pl_qkv1.smem);
  if (!arc) arc = set_smem_attr<MODE_RESID, 1>(std::max(m->pl_wo1.smem, m->pl_down1.smem));
  if (!arc) arc = set_smem_attr<MODE_GATEUP, 1>(m->pl_gu1.smem);
  if (!arc) arc = set_smem_attr<MODE_HEAD, 1>(m->pl_head1.smem);
  if (!arc) arc = set_smem_attr<MODE_STORE, 1>(std::max(m->pl_wo1.smem, m->pl_down1.smem));
  if (!arc) arc = set_smem_attr<MODE_QKV, PREFILL_TILE>(m->pl_qkvT.smem);
  if (!arc) arc = set_smem_attr<MODE_RESID, PREFILL_TILE>(std::max(m->pl_woT.smem, m->pl_downT.smem));
  if (!arc) arc = set_smem_attr<MODE_GATEUP, PREFILL_TILE>(m->pl_guT.smem);
  if (!arc && m->max_batch > 1) {
    // 16 sequences per weight pass, or 8 where 16 activation rows of the
    // widest K (ffn_down) do not fit shared memory
    auto plans = [&](int nb) {
      m->pl_qkvB = make_plan(qkv_rows, 2, qkv_rb, 1, m->n_embd, nb, true, nsm, SMEM_LIMIT, m->q80);
      m->pl_woB = make_plan(m->n_embd, 1, wo_rb, 1, (int)QN, nb, false, nsm, SMEM_LIMIT, m->q80);
      m->pl_guB = make_plan(m->n_ff, 1, gu_rb, 1, m->n_embd, nb, true, nsm, SMEM_LIMIT, m->q80);
      m->pl_downB = make_plan(m->n_embd, 1, dn_rb, 1, m->n_ff, nb, false, nsm, SMEM_LIMIT, m->q80);
      m->pl_headB = make_plan(m->output.rows, 1, m->output.row_bytes, 1, m->n_embd, nb, true, nsm, SMEM_LIMIT, m->q80);
      for (const Plan* pl : {&m->pl_qkvB, &m->pl_woB, &m->pl_guB, &m->pl_downB, &m->pl_headB})
        if (pl->smem > SMEM_LIMIT) return false;
      return true;
    };
    m->batch_nb = BATCH_NB;
    if (!plans(BATCH_NB)) {
      m->batch_nb = BATCH_NB_WIDE;
      if (!plans(BATCH_NB_WIDE)) { free_model(m); return fail(ARMAI_E_INVALID, "model rows too wide for batched decode"); }
    }
    // ranks other than 0 of a tensor-parallel model store their row-split
    // partial sums with MODE_STORE
    auto attrs = [&](auto nbc) {
      constexpr int NB = decltype(nbc)::value;
      int a = set_smem_attr<MODE_QKV, NB>(m->pl_qkvB.smem);
      if (!a) a = set_smem_attr<MODE_RESID, NB>(std::max(m->pl_woB.smem, m->pl_downB.smem));
      if (!a) a = set_smem_attr<MODE_GATEUP, NB>(m->pl_guB.smem);
      if (!a) a = set_smem_attr<MODE_HEAD, NB>(m->pl_headB.smem);
      if (!a) a = set_smem_attr<MODE_STORE, NB>(std::max(m->pl_woB.smem, m->pl_downB.smem));
      return a;
    };
    arc = m->batch_nb == BATCH_NB ? attrs(std::integral_constant<int, BATCH_NB>{})
                                  : attrs(std::integral_constant<int, BATCH_NB_WIDE>{});
    if (!arc) {
      const cudaError_t he = cudaMallocHost(&m->h_btok, (size_t)m->max_batch * 4);
      if (he != cudaSuccess) arc = cuda_fail(he, "cudaMallocHost", __FILE__, __LINE__);
    }
  }
  if (arc) { free_model(m); return arc; }
  m->attn_smem = attn_smem_floats(m->head_dim) * 4;
  m->n_kernels_step = 2 + 5 * m->n_layer;
  if (m->use_mega) {
    int src = setup_mega(m, nsm);
    if (src != ARMAI_OK) { free_model(m); return src; }
    m->n_kernels_step = 1;
  }
  LOAD_CUDA(cudaStreamSynchronize(m->stream));

  // capture the decode step (the per-kernel chain only: the persistent
  // kernel is a single launch, and as a graph node it ran slower)
  if (m->use_graph && !m->use_mega) {
    cudaGraph_t gr = nullptr;
    LOAD_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int erc = enqueue_decode_step(m);
    cudaError_t ec = cudaStreamEndCapture(m->stream, &gr);
    if (erc != ARMAI_OK || ec != cudaSuccess) {
      if (gr) cudaGraphDestroy(gr);
      int r = erc != ARMAI_OK ? erc : cuda_fail(ec, "cudaStreamEndCapture", __FILE__, __LINE__);
      free_model(m);
      return r;
    }
    ce = cudaGraphInstantiate(&m->graph, gr, 0);
    cudaGraphDestroy(gr);
    if (ce != cudaSuccess) { int r = cuda_fail(ce, "cudaGraphInstantiate", __FILE__, __LINE__); free_model(m); return r; }
  }
  size_t fb = 0, tb = 0;
  cudaMemGetInfo(&fb, &tb);
  m->device_bytes = arena + 2 * kv_bytes;
  *out = m;
  return ARMAI_OK;
#undef LOAD_CUDA
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" void armai_llama_default_opts(armai_llama_opts* o) {
  std::memset(o, 0, sizeof *o);
  o->device = 0;
  o->max_seq_len = 4096;
  o->kv_f16 = 0;
  o->max_batch = 1;
  o->use_graph = 1;
  o->use_pdl = 1;
  o->tp_size = 1;
  o->tp_rank = 0;
}

extern "C" int armai_llama_load(const char* path, const armai_llama_opts* opts, armai_llama** out) {
  if (!out) return fail(ARMAI_E_INVALID, "load: null output handle");
  *out = nullptr;
  if (!path || !*path) return fail(ARMAI_E_IO, "open failed: empty path");
  return load_model(path, opts, out);
}

extern "C" void armai_llama_free(armai_llama* m) { free_model(m); }

extern "C" int armai_llama_get_info(const armai_llama* m, armai_llama_info* info) {
  if (!m || !info) return fail(ARMAI_E_INVALID, "get_info: null argument");
  info->n_layer = m->n_layer;
  info->n_embd = m->n_embd;
  info->n_ff = m->n_ff;
  info->n_head = m->n_head;
  info->n_head_kv = m->n_head_kv;
  info->head_dim = m->head_dim;
  info->n_vocab = m->n_vocab;
  info->max_seq_len = m->max_seq;
  info->rms_eps = m->eps;
  info->rope_theta = m->rope_base;
  info->weight_bytes = m->weight_bytes_per_token;
  info->device_bytes = (int64_t)m->device_bytes;
  info->n_kernels_per_step = m->n_kernels_step;
  info->kv_f16 = m->kv_f16;
  return ARMAI_OK;
}

extern "C" int armai_llama_forward(armai_llama* m, const uint32_t* tokens, size_t n, size_t index_pos,
                                   float* logits, uint32_t* token) {
  if (!m || (!tokens && n)) return fail(ARMAI_E_INVALID, "forward: null argument");
  std::lock_guard<std::mutex> lk(m->mu);
  if (m->broken) return fail(ARMAI_E_DEVICE, "model is in an error state; reload it");
  ARMAI_CUDA(cudaSetDevice(m->device));
  ARMAI_TRY(forward_locked(m, tokens, (int)n, (int)index_pos));
  if (logits && m->tp > 1) {  // every rank's vocab rows, in rank order
    ARMAI_TRY(nccl_allgather_b32(m->logits, m->logits_all, (size_t)m->v_stride, m->comm, m->stream));
    ARMAI_CUDA(cudaMemcpyAsync(logits, m->logits_all, (size_t)m->n_vocab * 4, cudaMemcpyDeviceToHost, m->stream));
  } else if (logits) {
    ARMAI_CUDA(cudaMemcpyAsync(logits, m->logits, (size_t)m->n_vocab * 4, cudaMemcpyDeviceToHost, m->stream));
  }
  ARMAI_CUDA(cudaMemcpyAsync(m->h_tok, m->d_token, 4, cudaMemcpyDeviceToHost, m->stream));
  ARMAI_TRY(check_device_error(m));
  if (token) *token = m->h_tok[0];
  return ARMAI_OK;
}

extern "C" int armai_llama_generate(armai_llama* m, const uint32_t* prompt, size_t n_prompt,
                                    size_t max_new, const uint32_t* stop, size_t n_stop,
                                    armai_token_cb on_token, void* user, uint32_t* out,
                                    size_t* n_out, uint64_t* prefill_us, uint64_t* decode_us) {
  if (!m || !n_out || !prefill_us || !decode_us) return fail(ARMAI_E_INVALID, "generate: null argument");
  *n_out = 0;
  *prefill_us = 0;
  *decode_us = 0;
  if (max_new == 0 || n_prompt == 0) return ARMAI_OK;  // llama_candle.rs:76-78
  if (!prompt || !out) return fail(ARMAI_E_INVALID, "generate: null prompt or output buffer");
  std::lock_guard<std::mutex> lk(m->mu);  // llama_candle.rs:80 (Mutex per model)
  if (m->broken) return fail(ARMAI_E_DEVICE, "model is in an error state; reload it");
  ARMAI_CUDA(cudaSetDevice(m->device));
  if (n_prompt + max_new - 1 > (size_t)m->max_seq)
    return fail(ARMAI_E_RANGE, "generate: prompt + max_new - 1 = " + std::to_string(n_prompt + max_new - 1) +
                                   " positions exceed the rotary table (max_seq_len " + std::to_string(m->max_seq) + ")");
  auto is_stop = [&](uint32_t t) {
    for (size_t i = 0; i < n_stop; i++)
      if (stop[i] == t) return true;
    return false;
  };
  using clk = std::chrono::steady_clock;
  const auto t0 = clk::now();
  ARMAI_TRY(forward_locked(m, prompt, (int)n_prompt, 0));
  ARMAI_CUDA(cudaMemcpyAsync(m->h_tok, m->d_token, 4, cudaMemcpyDeviceToHost, m->stream));
  ARMAI_TRY(wait_done(m));
  *prefill_us = (uint64_t)std::chrono::duration_cast<std::chrono::microseconds>(clk::now() - t0).count();
  uint32_t next = m->h_tok[0];
  size_t n = 0;
  out[n++] = next;
  if (on_token) on_token(user, next);
  const auto t1 = clk::now();
  // Decode: step i consumes token i-1 (already on the device) and produces
  // token i. Step i+1 is enqueued before token i reaches the host, so the
  // GPU never idles on the host round trip; its result is discarded if token
  // i turns out to be a stop token (the reference stops before running it).
  const int RING = 8;
  cudaEvent_t ev[RING];
  for (int i = 0; i < RING; i++) cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
  int rc = ARMAI_OK;
  auto launch_step = [&](size_t i) -> int {
    ARMAI_TRY(run_decode_step(m));
    ARMAI_CUDA(cudaMemcpyAsync(&m->h_tok[i % RING], m->d_token, 4, cudaMemcpyDeviceToHost, m->stream));
    ARMAI_CUDA(cudaEventRecord(ev[i % RING], m->stream));
    return ARMAI_OK;
  };
  if (max_new > 1 && !is_stop(next)) rc = launch_step(1);
  for (size_t i = 1; i < max_new && rc == ARMAI_OK; i++) {
    if (is_stop(next)) break;  // llama_candle.rs:110
    if (i + 1 < max_new) {
      rc = launch_step(i + 1);
      if (rc) break;
    }
    rc = wait_done(m, ev[i % RING]);
    if (rc) break;
    next = m->h_tok[i % RING];
    out[n++] = next;
    if (on_token) on_token(user, next);
  }
  {
    const int wr = wait_done(m);  // steps launched ahead
    if (rc == ARMAI_OK) rc = wr;
  }
  *decode_us = (uint64_t)std::chrono::duration_cast<std::chrono::microseconds>(clk::now() - t1).count();
  for (int i = 0; i < RING; i++) cudaEventDestroy(ev[i]);
  m->kv_len = (int)(n_prompt + n - 1);
  *n_out = n;
  if (rc != ARMAI_OK) return rc;
  return check_device_error(m);
}

extern "C" int armai_llama_generate_batch(armai_llama* m, const uint32_t* prompts, const size_t* n_prompt,
                                          size_t n_seq, size_t max_new, const uint32_t* stop, size_t n_stop,
                                          uint32_t* out, size_t* n_out, uint64_t* prefill_us,
                                          uint64_t* decode_us) {
  if (!m || (n_seq && (!n_prompt || !n_out)) || !prefill_us || !decode_us || (n_stop && !stop))
    return fail(ARMAI_E_INVALID, "generate_batch: bad argument");
  *prefill_us = *decode_us = 0;
  for (size_t s = 0; s < n_seq; s++) n_out[s] = 0;
  if (!n_seq || !max_new) return ARMAI_OK;
  if (!out || !prompts) return fail(ARMAI_E_INVALID, "generate_batch: bad argument");
  if (m->max_batch == 1 && n_seq == 1)  // no batch slots: the single-sequence path
    return armai_llama_generate(m, prompts, n_prompt[0], max_new, stop, n_stop, nullptr, nullptr, out, n_out,
                                prefill_us, decode_us);
  std::lock_guard<std::mutex> lk(m->mu);
  if (m->broken) return fail(ARMAI_E_DEVICE, "model is in an error state; reload it");
  if ((int64_t)n_seq > m->max_batch)
    return fail(ARMAI_E_INVALID, "generate_batch: " + std::to_string(n_seq) +
                                     " sequences but the model was loaded with max_batch " +
                                     std::to_string(m->max_batch));
  size_t off = 0;
  for (size_t s = 0; s < n_seq; s++) {
    for (size_t i = 0; i < n_prompt[s]; i++)
      if (prompts[off + i] >= (uint32_t)m->n_vocab)
        return fail(ARMAI_E_INVALID, "generate_batch: sequence " + std::to_string(s) + ": token id " +
                                         std::to_string(prompts[off + i]) + " out of range for vocab " +
                                         std::to_string(m->n_vocab));
    if (n_prompt[s] && n_prompt[s] + max_new - 1 > (size_t)m->max_seq)
      return fail(ARMAI_E_RANGE, "generate_batch: sequence " + std::to_string(s) + ": " +
                                     std::to_string(n_prompt[s]) + " prompt + " + std::to_string(max_new) +
                                     " new tokens exceed max_seq_len " + std::to_string(m->max_seq));
    off += n_prompt[s];
  }
  ARMAI_CUDA(cudaSetDevice(m->device));
  m->kv_len = -1;  // the single-sequence cache (slot 0) no longer continues
  const int n = (int)n_seq;
  // Prefill every sequence into its slot; empty prompts decode from token 0
  // at position 0 and their outputs are discarded.
  auto t0 = std::chrono::steady_clock::now();
  ARMAI_CUDA(cudaMemsetAsync(m->d_token, 0, (size_t)n * 4, m->stream));
  ARMAI_CUDA(cudaMemsetAsync(m->d_pos, 0, (size_t)n * 4, m->stream));
  off = 0;
  for (int s = 0; s < n; s++) {
    if (n_prompt[s]) ARMAI_TRY(enqueue_prefill(m, prompts + off, (int)n_prompt[s], s));
    off += n_prompt[s];
  }
  ARMAI_TRY(check_device_error(m));
  auto t1 = std::chrono::steady_clock::now();
  std::vector<char> done(n, 0);
  int live = 0;
  for (int s = 0; s < n; s++) live += (done[s] = n_prompt[s] == 0) ? 0 : 1;
  auto record = [&]() {
    for (int s = 0; s < n; s++) {
      if (done[s]) continue;
      const uint32_t t = m->h_btok[s];
      out[(size_t)s * max_new + n_out[s]++] = t;
      bool hit = n_out[s] >= max_new;
      for (size_t k = 0; k < n_stop && !hit; k++) hit = stop[k] == t;
      if (hit) { done[s] = 1; live--; }
    }
  };
  ARMAI_CUDA(cudaMemcpyAsync(m->h_btok, m->d_token, (size_t)n * 4, cudaMemcpyDeviceToHost, m->stream));
  ARMAI_TRY(wait_done(m));
  record();
  while (live > 0) {
    ARMAI_TRY(enqueue_batch_step(m, n));
    ARMAI_CUDA(cudaMemcpyAsync(m->h_btok, m->d_token, (size_t)n * 4, cudaMemcpyDeviceToHost, m->stream));
    ARMAI_TRY(check_device_error(m));
    record();
  }
  auto t2 = std::chrono::steady_clock::now();
  *prefill_us = (uint64_t)std::chrono::duration_cast<std::chrono::microseconds>(t1 - t0).count();
  *decode_us = (uint64_t)std::chrono::duration_cast<std::chrono::microseconds>(t2 - t1).count();
  return ARMAI_OK;
}

extern "C" int armai_llama_bench_decode(armai_llama* m, int32_t n_steps, float* ms) {
  if (!m || !ms || n_steps <= 0) return fail(ARMAI_E_INVALID, "bench_decode: bad argument");
  std::lock_guard<std::mutex> lk(m->mu);
  ARMAI_CUDA(cudaSetDevice(m->device));
  if (m->kv_len + n_steps > m->max_seq) return fail(ARMAI_E_RANGE, "bench_decode: steps exceed max_seq_len");
  cudaEvent_t a, b;
  ARMAI_CUDA(cudaEventCreate(&a));
  ARMAI_CUDA(cudaEventCreate(&b));
  ARMAI_CUDA(cudaEventRecord(a, m->stream));
  for (int i = 0; i < n_steps; i++) ARMAI_TRY(run_decode_step(m));
  ARMAI_CUDA(cudaEventRecord(b, m->stream));
  ARMAI_TRY(wait_done(m, b));
  ARMAI_CUDA(cudaEventElapsedTime(ms, a, b));
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  m->kv_len += n_steps;
  return check_device_error(m);
}

extern "C" int armai_llama_bench_kernel(armai_llama* m, int32_t kind, int32_t rounds, float* ms_per_launch,
                                        int64_t* bytes_per_launch) {
  if (!m || !ms_per_launch || !bytes_per_launch || rounds <= 0 || kind < 0 || kind > 5)
    return fail(ARMAI_E_INVALID, "bench_kernel: bad argument");
  std::lock_guard<std::mutex> lk(m->mu);
  ARMAI_CUDA(cudaSetDevice(m->device));
  const bool pdl = m->use_pdl;
  m->use_pdl = false;
  int64_t bytes = 0;
  int launches = 0;
  auto one = [&](int l) -> cudaError_t {
    const Layer& L = m->layers[l];
    switch (kind) {
      case 0: bytes += (int64_t)L.wg.rows * L.wg.row_bytes + (int64_t)L.wu.rows * L.wu.row_bytes;
              return launch_gateup<1>(m, m->pl_gu1, l, m->x, m->h);
      case 1: bytes += (int64_t)L.wq.rows * L.wq.row_bytes + (int64_t)L.wk.rows * L.wk.row_bytes +
                       (int64_t)L.wv.rows * L.wv.row_bytes;
              return launch_qkv<1>(m, m->pl_qkv1, l, m->x, m->q, m->d_pos, 0);
      case 2: bytes += (int64_t)L.wo.rows * L.wo.row_bytes;
              return launch_resid<1>(m, m->pl_wo1, L.wo, m->y, m->x);
      case 3: bytes += (int64_t)L.wd.rows * L.wd.row_bytes;
              return launch_resid<1>(m, m->pl_down1, L.wd, m->h, m->x);
      case 4: bytes += (int64_t)m->output.rows * m->output.row_bytes;
              return launch_head<1>(m, m->pl_head1, m->x, m->d_pos, nullptr, m->d_token);
      default: return launch_attn(m, l, m->q, m->y, m->d_pos, 1, 0);
    }
  };
  cudaEvent_t a, b;
  ARMAI_CUDA(cudaEventCreate(&a));
  ARMAI_CUDA(cudaEventCreate(&b));
  int rc = ARMAI_OK;
  for (int l = 0; l < m->n_layer && rc == ARMAI_OK; l++)  // warm-up round
    if (one(l) != cudaSuccess) rc = fail(ARMAI_E_CUDA, "bench_kernel: launch failed");
  bytes = 0;
  cudaEventRecord(a, m->stream);
  for (int r = 0; r < rounds && rc == ARMAI_OK; r++)
    for (int l = 0; l < (kind == 4 ? 1 : m->n_layer) && rc == ARMAI_OK; l++) {
      if (one(l) != cudaSuccess) rc = fail(ARMAI_E_CUDA, "bench_kernel: launch failed");
      launches++;
    }
  cudaEventRecord(b, m->stream);
  m->use_pdl = pdl;
  if (rc != ARMAI_OK) { cudaEventDestroy(a); cudaEventDestroy(b); return rc; }
  ARMAI_TRY(wait_done(m, b));
  float ms = 0.f;
  ARMAI_CUDA(cudaEventElapsedTime(&ms, a, b));
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  *ms_per_launch = ms / (float)launches;
  *bytes_per_launch = bytes / launches;
  return check_device_error(m);
}

extern "C" int armai_llama_trace_decode(armai_llama* m, uint64_t* out, size_t cap, int32_t* n_phases,
                                        int32_t* n_ctas) {
  if (!m || !out || !n_phases || !n_ctas) return fail(ARMAI_E_INVALID, "trace_decode: bad argument");
  std::lock_guard<std::mutex> lk(m->mu);
  if (m->broken) return fail(ARMAI_E_DEVICE, "model is in an error state; reload it");
  if (!m->use_mega) return fail(ARMAI_E_INVALID, "trace_decode: needs the persistent decode kernel");
  const size_t n = (size_t)(m->mk.n_ph + 1) * m->mk_grid * MK_TRACE_SLOTS;
  if (cap < n) return fail(ARMAI_E_RANGE, "trace_decode: buffer holds " + std::to_string(cap) +
                                              " stamps, needs " + std::to_string(n));
  if (m->kv_len + 1 > m->max_seq) return fail(ARMAI_E_RANGE, "trace_decode: KV cache is full");
  ARMAI_CUDA(cudaSetDevice(m->device));
  unsigned long long* d = nullptr;
  ARMAI_CUDA(cudaMalloc(&d, n * 8));
  cudaError_t e = cudaMemsetAsync(d, 0, n * 8, m->stream);
  if (e == cudaSuccess) {
    m->mk.trace = d;
    e = launch_mega(m);
    m->mk.trace = nullptr;
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(out, d, n * 8, cudaMemcpyDeviceToHost, m->stream);
  int wrc = e == cudaSuccess ? wait_done(m) : ARMAI_OK;
  cudaFree(d);
  if (e != cudaSuccess) return cuda_fail(e, "trace_decode", __FILE__, __LINE__);
  ARMAI_TRY(wrc);
  m->kv_len += 1;
  *n_phases = m->mk.n_ph + 1;
  *n_ctas = m->mk_grid;
  return check_device_error(m);
}

extern "C" int armai_llama_test_stall(armai_llama* m, int32_t phase, uint32_t poll_limit) {
  if (!m) return fail(ARMAI_E_INVALID, "test_stall: null model");
  std::lock_guard<std::mutex> lk(m->mu);
  if (!m->use_mega) return fail(ARMAI_E_INVALID, "test_stall: needs the persistent decode kernel");
  if (phase < 0 || phase >= m->mk.n_ph) return fail(ARMAI_E_RANGE, "test_stall: no such phase");
  m->mk.test_stall_phase = phase;
  m->mk.poll_limit = poll_limit ? poll_limit : MK_BAR_LIMIT;
  return ARMAI_OK;
}

extern "C" int armai_nccl_unique_id(void* out128) {
  if (!out128) return fail(ARMAI_E_INVALID, "nccl_unique_id: null argument");
  return nccl_unique_id(out128);
}
