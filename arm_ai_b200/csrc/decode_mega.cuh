// decode_mega.cuh — persistent single-launch decode step (sm_100a).
//
// One CTA per SM runs the whole decode step of one sequence:
//   for each layer: QKV (+RoPE, KV append) | attention | attn_output (+residual)
//                   | gate/up (+SiLU*up) | ffn_down (+residual)
//   then output_norm + output head + greedy argmax.
// There is no grid barrier. Every value a phase hands to the next one (q, the
// new K/V row, the attention output y, h = silu(gate) * up, the attn_output /
// ffn_down row sums) is a 64-bit word: a generation tag in the low half, the
// f32 bits in the high half, written by one single-copy-atomic store. A
// reader polls the words it needs until they carry the tag of this step's
// producing phase (generation = step * (phases + 1) + phase + 1), so each
// phase starts as soon as its own inputs exist. Every CTA keeps the whole
// residual stream x in shared memory and folds the row sums of attn_output /
// ffn_down into it itself (tensor parallelism: the sums of every rank, in
// rank order, from slots that each rank writes into every rank's memory).
//
// Buffers are reused from layer to layer (q, K/V row, y, h) or by parity (row
// sums of attn_output vs ffn_down). That is safe because every CTA owns rows
// in every matvec phase and reads its whole input vector: a phase's output
// can only be overwritten after every CTA has read it, since the overwriting
// phase depends on outputs of all CTAs of a later phase.
//
// Warp 0 is a producer: one lane walks the same phase/chunk sequence as the
// consumers and streams every weight row this CTA owns HBM -> shared memory
// with cp.async.bulk into a ring of stages (full/empty mbarriers). It runs
// ahead across phase boundaries, so weight traffic continues while the
// consumers wait for their inputs or run attention. The other MK_CW warps are
// consumers: they build the Q8_K activation of the phase (rmsnorm +
// quantisation), run the register-slice dot products on the staged rows, and
// apply the epilogue.
//
// Every wait is bounded and checks the device error word, so a stuck copy or
// a CTA that left early ends the launch with an error instead of a hang.
#pragma once

#include "llama_kernels.cuh"

namespace armai {

// Consumer warps: 11 leave each thread up to 168 registers (12 warps at one
// CTA per SM); at 15 the compiler squeezed the step into 128 and it ran about
// 4 % slower.
#ifndef ARMAI_MK_CW
#define ARMAI_MK_CW 11
#endif
constexpr int MK_CW = ARMAI_MK_CW;             // consumer warps
constexpr int MK_THREADS = 32 * (1 + MK_CW);
constexpr int MK_CT = 32 * MK_CW;             // consumer threads
constexpr uint32_t MK_STAGE = 32 * 1024;
constexpr int MK_MAX_NS = 6;
constexpr uint32_t MK_BAR_LIMIT = 1u << 24;   // grid-barrier polls before giving up
constexpr int MK_ATT_PER_HEAD_MAX_T = 512;    // attention unit per query head up to this context
constexpr int MK_REGJ = 2;                    // prologue blocks per warp kept in registers

enum { PH_QKV = 0, PH_ATTN = 1, PH_WO = 2, PH_GATEUP = 3, PH_DOWN = 4, PH_HEAD = 5 };

struct MkPhase {
  int kind, layer;
  Seg seg[3];
  int nseg;
  int total_rows;     // QKV: q+k+v rows; GATEUP: rows of each matrix; else rows
  int rows_per_cta;   // multiple of 2 for QKV
  int chunk_rows;     // multiple of 2 for QKV
  int K, nb;
  int acts;           // activations the rows need: 1 Q8_K (k-quants), 2 Q8_0 (legacy types)
  const float* gamma; // rmsnorm weight, or nullptr
  float* out;         // HEAD: logits (nullptr: not kept)
  void* kc;           // layer KV cache
  void* vc;
};

constexpr int MK_TP_MAX = 8;

struct MkParams {
  const MkPhase* ph;
  int n_ph;
  int ns;
  const uint8_t* embd;
  int embd_type, embd_row_bytes, n_embd;
  const float* cos_t;
  const float* sin_t;
  int hd, n_head, n_kv, max_seq, kv_f16;
  float eps;
  float att_scale;
  float* att_part;
  unsigned* att_cnt;
  // tagged words (see the top of this file)
  unsigned long long* fq;   // [n_head * hd] RoPE'd q
  unsigned long long* fkv;  // [2][n_kv][hd] this step's K and V rows (as the cache holds them)
  unsigned long long* fy;   // [n_head * hd] attention output
  unsigned long long* fh;   // [n_ff] silu(gate) * up
  float* am_val;
  int* am_idx;
  unsigned* am_cnt;
  uint32_t* token;
  int* pos;
  uint32_t* err;
  // Polls of a tagged word before a wait gives up (sets the error word and
  // lets the launch end); MK_BAR_LIMIT unless a test shortens it.
  uint32_t poll_limit;
  // Test injection: the phase whose outputs are never published (-1: none),
  // so that its consumers' bounded waits run out.
  int test_stall_phase;
  unsigned long long* trace;  // nullptr, or [n_ph][grid][MK_TRACE_SLOTS] globaltimer stamps
  size_t off_bars, off_act_qs, off_act_d, off_act_bs, off_red, off_att;  // smem layout
  size_t off_act0_qs, off_act0_d, off_act0_s;  // Q8_0 activation (0: no phase needs one)
  int kmax;
  size_t off_xrep;  // smem: this CTA's copy of the residual stream x [n_embd]
  unsigned long long* epoch;            // decode steps completed (generation base)
  // Row sums of attn_output (parity 1) / ffn_down (parity 0): rank k's slots
  // [2][tp][n_embd]; tp = 1 is one local array. Tensor parallelism maps the
  // other ranks' arrays through CUDA IPC.
  int tp, tp_rank, v0;                  // v0: first vocab row of this rank
  unsigned long long* xslot[MK_TP_MAX];
  uint32_t* hslot[MK_TP_MAX];           // rank k's head winners [2][tp][2] (tp > 1)
  unsigned long long* hctr[MK_TP_MAX];  // rank k's head counter (tp > 1)
};

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Phase timeline (profiling), stamped by the first consumer thread: slot 0
// phase start (grid barrier passed), 1 activation built, 2 phase done,
// 3 producer issued the phase's first chunk, 4 first chunk's data ready,
// 5 first chunk computed, 6 prologue's first pass done, 7 rms scale known,
// 8 / 9 first unit's dot products / epilogue done.
constexpr int MK_TRACE_SLOTS = 12;
__device__ __forceinline__ void mk_stamp(const MkParams& p, int phase, int slot) {
  if (p.trace) p.trace[((size_t)phase * gridDim.x + blockIdx.x) * MK_TRACE_SLOTS + slot] = global_ns();
}

__device__ __forceinline__ void prefetch_l1(const void* ptr) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(ptr));
}

__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys_add64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded wait until *ctr >= target (system scope); false (and the error flag)
// when it gives up.
__device__ __forceinline__ bool wait_ge_sys(const unsigned long long* ctr, unsigned long long target, uint32_t* err) {
  for (uint32_t it = 0;; ++it) {
    if (ld_acquire_sys_u64(ctr) >= target) return true;
    if (it > 32) __nanosleep(64);
    if ((it & 255) == 0 && *reinterpret_cast<const volatile uint32_t*>(err) != 0u) return false;
    if (it > MK_BAR_LIMIT) { atomicOr(err, DEVERR_COUNTER_TIMEOUT); return false; }
  }
}

__device__ __forceinline__ bool dev_failed(const uint32_t* err) {
  return *reinterpret_cast<const volatile uint32_t*>(err) != 0u;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bounded mbarrier wait that also gives up when another CTA flagged an error.
__device__ __forceinline__ bool mk_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t* iters = nullptr) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < WAIT_LIMIT; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    if (iters) *iters = i + 1;
    if (ok) return true;
    if (i > 8) {
      if ((i & 63) == 0 && dev_failed(err)) return false;
      __nanosleep(128);
    }
  }
  atomicOr(err, DEVERR_MBAR_TIMEOUT);
  return false;
}

__device__ __forceinline__ int mode_of(int kind) {
  return kind == PH_QKV ? MODE_QKV : kind == PH_GATEUP ? MODE_GATEUP : kind == PH_HEAD ? MODE_HEAD
                                                                                     : MODE_RESID;
}

// Rows [r0, r1) of this CTA: the phase's units (QKV: RoPE pairs of rows,
// else single rows) split as evenly as possible over the grid. The grid is
// no larger than the smallest phase's unit count, so every CTA owns rows in
// every matvec phase (which the buffer reuse relies on).
__device__ __forceinline__ void phase_rows(const MkPhase& ph, int& r0, int& r1) {
  // 32-bit arithmetic: units (at most a vocabulary's rows) x grid stays far
  // below 2^31, and a 64-bit division is a long software routine
  const int unit = ph.kind == PH_QKV ? 2 : 1;
  const int U = (ph.total_rows + unit - 1) / unit, G = gridDim.x, b = blockIdx.x;
  r0 = min((b * U / G) * unit, ph.total_rows);
  r1 = min(((b + 1) * U / G) * unit, ph.total_rows);
}

// ---------------------------------------------------------------------------
// Producer: one lane streams this CTA's rows of every weight phase.
// ---------------------------------------------------------------------------
// Bounded wait for a copy's completion that does not give up early when
// another CTA failed: a CTA must not exit with its own copies in flight.
__device__ __forceinline__ void mk_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  for (uint32_t i = 0; i < WAIT_LIMIT; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    if (ok) return;
    if (i > 8) __nanosleep(128);
  }
}

__device__ void mk_producer(const MkParams& p, uint8_t* smem) {
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bars);
  uint64_t* empty = full + MK_MAX_NS;
  const uint64_t pol = l2_evict_first_policy();
  int sidx = 0;
  // On every exit (normal, or a wait that gave up): the stages issued last
  // have landed before this thread leaves (normally they were consumed).
  struct Drain {
    uint64_t* full;
    const int& sidx;
    int ns;
    __device__ ~Drain() {
      for (int j = sidx > ns ? sidx - ns : 0; j < sidx; j++) mk_drain(&full[j % ns], (uint32_t)((j / ns) & 1));
    }
  } drain{full, sidx, p.ns};
  for (int i = 0; i < p.n_ph; i++) {
    const MkPhase& ph = p.ph[i];
    if (ph.kind == PH_ATTN) continue;
    int r0, r1;
    phase_rows(ph, r0, r1);
    const int mode = mode_of(ph.kind);
    for (int c0 = r0; c0 < r1; c0 += ph.chunk_rows) {
      const int c1 = min(c0 + ph.chunk_rows, r1);
      const int s = sidx % p.ns;
      if (sidx >= p.ns && !mk_wait(&empty[s], (uint32_t)(((sidx / p.ns) - 1) & 1), p.err)) return;
      if (c0 == r0) mk_stamp(p, i, 3);
      Part parts[3];
      if (mode == MODE_QKV) make_parts<MODE_QKV>(ph.seg, ph.nseg, c0, c1, parts);
      else if (mode == MODE_GATEUP) make_parts<MODE_GATEUP>(ph.seg, ph.nseg, c0, c1, parts);
      else make_parts<MODE_RESID>(ph.seg, ph.nseg, c0, c1, parts);
      fence_proxy_async();
      issue_parts(ph.seg, parts, smem + (size_t)s * MK_STAGE, &full[s], pol);
      sidx++;
    }
  }
}

// Values [8 lane, 8 lane + 8) of super-block j of the current token's
// embedding row (BlockQ4K / BlockQ6K::to_float). Inlined: out of line, the
// returned struct went through local memory and dragged the prologue's
// value array there with it.
struct F8 {
  float v[8];
};
__device__ __forceinline__ F8 mk_embed_vals(const MkParams& p, int j, int lane, int nb) {
  F8 out;
  const uint32_t tok = min(__ldcg(p.token), (uint32_t)(0x7fffffff));
  dequant8(p.embd_type, p.embd + (int64_t)tok * p.embd_row_bytes, nb, j, lane, out.v);
  return out;
}

// ---------------------------------------------------------------------------
// Consumer prologue: Q8_K activation of the phase input (optionally rmsnorm).
// Layer 0's QKV reads the token's embedding row (dequantised here by every
// CTA into its copy of x).
// ---------------------------------------------------------------------------
// Tagged words: generation tag (low half) | f32 bits (high half), each
// stored by one single-copy-atomic 64-bit store, so a reader that sees the
// tag sees the value stored with it. Local words use gpu scope; the row-sum
// slots, which other ranks write over NVLink, system scope.
__device__ __forceinline__ unsigned long long tag_word(uint32_t tag, float v) {
  return (unsigned long long)tag | ((unsigned long long)__float_as_uint(v) << 32);
}
__device__ __forceinline__ float word_val(unsigned long long w) { return __uint_as_float((uint32_t)(w >> 32)); }
__device__ __forceinline__ void st_word_gpu(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_word_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Two words per load; each of the pair is read atomically.
template <bool SYS>
__device__ __forceinline__ void ld_words2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
  if constexpr (SYS)
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
  else
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
template <bool SYS>
__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* p) {
  unsigned long long v;
  if constexpr (SYS)
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  else
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Bounded poll: false (and the error flag) when it gives up or another CTA
// failed.
__device__ __forceinline__ bool poll_continue(uint32_t it, uint32_t* err, uint32_t limit) {
  if (it > limit || (((it & 255) == 255) && dev_failed(err))) {
    atomicOr(err, DEVERR_COUNTER_TIMEOUT);
    return false;
  }
  if (it > 4) __nanosleep(20);
  return true;
}
// N (even) consecutive words (16-byte aligned) carrying tag `want`.
template <bool SYS, int N>
__device__ __forceinline__ void wait_words(const unsigned long long* p, uint32_t want, unsigned long long (&w)[N],
                                           uint32_t* err, uint32_t limit) {
#pragma unroll
  for (int e = 0; e < N; e += 2) ld_words2<SYS>(p + e, w[e], w[e + 1]);
  for (uint32_t it = 0;; ++it) {
    bool ok = true;
#pragma unroll
    for (int e = 0; e < N; e++) ok &= (uint32_t)w[e] == want;
    if (ok || !poll_continue(it, err, limit)) return;
#pragma unroll
    for (int e = 0; e < N; e += 2)
      if ((uint32_t)w[e] != want || (uint32_t)w[e + 1] != want) ld_words2<SYS>(p + e, w[e], w[e + 1]);
  }
}
// N (even) consecutive words at each of two addresses, all carrying tag
// `want`: both sets' loads are in flight together (one round trip for two
// ranks' row sums instead of two).
template <bool SYS, int N>
__device__ __forceinline__ void wait_words_pair(const unsigned long long* pa, const unsigned long long* pb,
                                                uint32_t want, unsigned long long (&wa)[N],
                                                unsigned long long (&wb)[N], uint32_t* err, uint32_t limit) {
#pragma unroll
  for (int e = 0; e < N; e += 2) {
    ld_words2<SYS>(pa + e, wa[e], wa[e + 1]);
    ld_words2<SYS>(pb + e, wb[e], wb[e + 1]);
  }
  for (uint32_t it = 0;; ++it) {
    bool ok = true;
#pragma unroll
    for (int e = 0; e < N; e++) ok &= ((uint32_t)wa[e] == want) & ((uint32_t)wb[e] == want);
    if (ok || !poll_continue(it, err, limit)) return;
#pragma unroll
    for (int e = 0; e < N; e += 2) {
      if ((uint32_t)wa[e] != want || (uint32_t)wa[e + 1] != want) ld_words2<SYS>(pa + e, wa[e], wa[e + 1]);
      if ((uint32_t)wb[e] != want || (uint32_t)wb[e + 1] != want) ld_words2<SYS>(pb + e, wb[e], wb[e + 1]);
    }
  }
}
// One word carrying tag `want`; its value.
template <bool SYS>
__device__ __forceinline__ float wait_word(const unsigned long long* p, uint32_t want, uint32_t* err,
                                           uint32_t limit) {
  unsigned long long w = ld_word<SYS>(p);
  for (uint32_t it = 0; (uint32_t)w != want && poll_continue(it, err, limit); ++it) w = ld_word<SYS>(p);
  return word_val(w);
}

// Values [8 lane, 8 lane + 8) of block j of phase i's input: the token
// embedding (layer 0's QKV), y (attn_output), h (ffn_down), or the residual
// stream x = this CTA's copy + the previous phase's row sums of every rank,
// added in rank order (QKV of later layers, gate/up, the head).
__device__ __forceinline__ F8 mk_load_vals_ool(const MkParams& p, const MkPhase& ph, int j, int lane, uint32_t want,
                                            const float* xrep) {
  float vv[8];
  if (ph.kind == PH_WO || ph.kind == PH_DOWN) {
    unsigned long long w[8];
    wait_words<false, 8>((ph.kind == PH_WO ? p.fy : p.fh) + j * QK_K + 8 * lane, want, w, p.err, p.poll_limit);
#pragma unroll
    for (int e = 0; e < 8; e++) vv[e] = word_val(w[e]);
  } else if (ph.kind == PH_QKV && ph.layer == 0) {
    const F8 e = mk_embed_vals(p, j, lane, ph.nb);
#pragma unroll
    for (int k = 0; k < 8; k++) vv[k] = e.v[k];
  } else {
    const int E = p.n_embd, par = ph.kind == PH_GATEUP ? 1 : 0;  // after attn_output : after ffn_down
    const float4* xr = reinterpret_cast<const float4*>(xrep + j * QK_K + 8 * lane);
    const float4 a = xr[0], b = xr[1];
    float acc[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const unsigned long long* sl = p.xslot[p.tp_rank] + (size_t)par * p.tp * E + j * QK_K + 8 * lane;
    int k = 0;
    for (; k + 1 < p.tp; k += 2) {  // two ranks' slots per round trip, added in rank order
      unsigned long long w[8], w2[8];
      wait_words_pair<true, 8>(sl + (size_t)k * E, sl + (size_t)(k + 1) * E, want, w, w2, p.err, p.poll_limit);
#pragma unroll
      for (int e = 0; e < 8; e++) acc[e] = __fadd_rn(__fadd_rn(acc[e], word_val(w[e])), word_val(w2[e]));
    }
    if (k < p.tp) {
      unsigned long long w[8];
      wait_words<true, 8>(sl + (size_t)k * E, want, w, p.err, p.poll_limit);
#pragma unroll
      for (int e = 0; e < 8; e++) acc[e] = __fadd_rn(acc[e], word_val(w[e]));
    }
#pragma unroll
    for (int e = 0; e < 8; e++) vv[e] = acc[e];
  }
  F8 r;
#pragma unroll
  for (int e = 0; e < 8; e++) r.v[e] = vv[e];
  return r;
}
__device__ __forceinline__ void mk_load_vals(const MkParams& p, const MkPhase& ph, int j, int lane, float (&vv)[8],
                                             uint32_t want, const float* xrep) {
  const F8 r = mk_load_vals_ool(p, ph, j, lane, want, xrep);
#pragma unroll
  for (int e = 0; e < 8; e++) vv[e] = r.v[e];
}

// Q8_K activation of phase i's input in shared memory (rmsnorm first when
// the phase has one). Phases that read x also store the new x into the CTA's
// copy. The first MK_REGJ blocks of a warp stay in registers between the two
// passes; any further ones (K > MK_REGJ * 256 * consumer warps) are read
// again in the second pass (from the copy of x, or the same tagged words).
__device__ void mk_build_act(const MkParams& p, const MkPhase& ph, int phase, uint8_t* smem,
                             const ActQ8 act, int cw, int lane, float* xrep, uint64_t* gbar, uint32_t gpar,
                             uint32_t want) {
  const int K = ph.K, nb = ph.nb;
  float* part = reinterpret_cast<float*>(smem + p.off_red) + 64;
  const bool norm = ph.gamma != nullptr;
  const bool is_x = ph.kind != PH_WO && ph.kind != PH_DOWN;
  // One call site per loader: every copy of the (inlined) loaders would be
  // instruction-cache footprint of every phase.
  float v[MK_REGJ][8];
  for (int j = cw, jj = 0; j < nb; j += MK_CW, jj++) {
    float vv[8];
    mk_load_vals(p, ph, j, lane, vv, want, xrep);
#pragma unroll
    for (int r = 0; r < MK_REGJ; r++)
      if (jj == r) {
#pragma unroll
        for (int k = 0; k < 8; k++) v[r][k] = vv[k];
      }
    if (is_x) {
      float4* xw = reinterpret_cast<float4*>(xrep + j * QK_K + 8 * lane);
      xw[0] = make_float4(vv[0], vv[1], vv[2], vv[3]);
      xw[1] = make_float4(vv[4], vv[5], vv[6], vv[7]);
    }
    if (norm) {
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < 8; k++) ss += vv[k] * vv[k];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) part[j] = ss;
    }
  }
  float m = 1.f;
  if (cw == 0 && lane == 0) mk_stamp(p, phase, 6);
  if (norm) {
    named_sync(1, MK_CT);
    // candle rms_norm: m = sqrt(sum2 / K + eps); block partials added in
    // block order by every thread (same value everywhere, no second barrier).
    float sum2 = 0.f;
    for (int j = 0; j < nb; j++) sum2 += part[j];
    m = __fsqrt_rn(__fadd_rn(__fdiv_rn(sum2, (float)K), p.eps));
    mk_wait(gbar, gpar, p.err);  // rmsnorm weights staged in shared memory
  }
  const float* gs = reinterpret_cast<const float*>(smem + p.off_att);
  if (cw == 0 && lane == 0) mk_stamp(p, phase, 7);
  for (int j = cw, jj = 0; j < nb; j += MK_CW, jj++) {
    float vv[8];
    if (jj < MK_REGJ) {
#pragma unroll
      for (int r = 0; r < MK_REGJ; r++)
        if (jj == r) {
#pragma unroll
          for (int k = 0; k < 8; k++) vv[k] = v[r][k];
        }
    } else if (is_x) {
      const float4* xr = reinterpret_cast<const float4*>(xrep + j * QK_K + 8 * lane);
      const float4 a = xr[0], b = xr[1];
      vv[0] = a.x; vv[1] = a.y; vv[2] = a.z; vv[3] = a.w;
      vv[4] = b.x; vv[5] = b.y; vv[6] = b.z; vv[7] = b.w;
    } else {  // y / h blocks beyond the register-held ones: read again
      unsigned long long w[8];
      wait_words<false, 8>((ph.kind == PH_WO ? p.fy : p.fh) + j * QK_K + 8 * lane, want, w, p.err, p.poll_limit);
#pragma unroll
      for (int e = 0; e < 8; e++) vv[e] = word_val(w[e]);
    }
    if (norm) {
      const float4* gr = reinterpret_cast<const float4*>(gs + j * QK_K + 8 * lane);
      const float4 g0 = gr[0], g1 = gr[1];
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
      for (int k = 0; k < 8; k++) vv[k] = __fmul_rn(__fdiv_rn(vv[k], m), g[k]);
    }
    if (ph.acts & 1) q8k_quant_block_warp(vv, lane, act.qs + j * QK_K, act.d + j, act.bs + j * 16, j & 7);
    if (ph.acts & 2) q80_quant_block_warp(vv, lane, act.qs0 + j * QK_K, act.d0 + 8 * j, act.s0 + 8 * j, j & 7);
  }
  named_sync(1, MK_CT);
}

// ---------------------------------------------------------------------------
// Consumer: dot products + epilogue of the staged chunks (chunk_units).
// ---------------------------------------------------------------------------
// Context of the persistent kernel's matvec phases.
struct MkCtx {
  const MkParams& p;
  const MkPhase& ph;
  int pos_v;
  int phase;
  uint32_t tag;  // generation of this phase's outputs
  __device__ const Seg& seg(int i) const { return ph.seg[i]; }
  __device__ int nb() const { return ph.nb; }
  __device__ float* out() const { return ph.out; }
  __device__ int qn() const { return ph.seg[0].rows; }
  __device__ int kn() const { return ph.seg[1].rows; }
  __device__ int hd() const { return p.hd; }
  __device__ int pos() const { return pos_v; }
  __device__ const float* cos_t() const { return p.cos_t; }
  __device__ const float* sin_t() const { return p.sin_t; }
  __device__ void stamp(int slot) const { mk_stamp(p, phase, slot); }
  __device__ bool stalled() const { return phase == p.test_stall_phase; }
  __device__ void put_q(int r, float a, float b) const {
    if (stalled()) return;
    st_word_gpu(p.fq + r, tag_word(tag, a));
    st_word_gpu(p.fq + r + 1, tag_word(tag, b));
  }
  // The cache row (read by later steps) and the tagged copy this step's
  // attention reads, with the cache's rounding.
  __device__ void put_kv(int which, int kvh, int dd, float a, float b) const {
    store_kv(which ? ph.vc : ph.kc, p.kv_f16, ((int64_t)kvh * p.max_seq + pos_v) * p.hd + dd, a, b);
    if (p.kv_f16) {
      a = __half2float(__float2half_rn(a));
      b = __half2float(__float2half_rn(b));
    }
    if (stalled()) return;
    unsigned long long* w = p.fkv + ((size_t)which * p.n_kv + kvh) * p.hd + dd;
    st_word_gpu(w, tag_word(tag, a));
    st_word_gpu(w + 1, tag_word(tag, b));
  }
  __device__ void put_h(int r, float v) const {
    if (!stalled()) st_word_gpu(p.fh + r, tag_word(tag, v));
  }
  // attn_output / ffn_down row r: this rank's sum into every rank's slot
  __device__ void resid_add(float*, int r, float v) const {
    const size_t off = ((size_t)(ph.kind == PH_WO ? 1 : 0) * p.tp + p.tp_rank) * p.n_embd + r;
    const unsigned long long w = tag_word(tag, v);
    if (stalled()) return;
    for (int k = 0; k < p.tp; k++) st_word_sys(p.xslot[k] + off, w);
  }
};

// ---------------------------------------------------------------------------
// The matvec phases share one copy of their code: the mode (q/k/v, residual,
// gate/up, head) and the weight types are runtime values. The whole decode
// step then executes a few tens of KB of instructions per layer, which stay
// in the SM's instruction cache; per-mode and per-type template copies made
// every phase start from cold code (an instruction fetched from outside the
// cache costs about ten cycles, so a latency-bound chain runs several times
// slower).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mk_parts(const MkPhase& ph, int mode, int c0, int c1, Part (&parts)[3]) {
  if (mode == MODE_QKV) make_parts<MODE_QKV>(ph.seg, ph.nseg, c0, c1, parts);
  else if (mode == MODE_GATEUP) make_parts<MODE_GATEUP>(ph.seg, ph.nseg, c0, c1, parts);
  else make_parts<MODE_RESID>(ph.seg, ph.nseg, c0, c1, parts);
}
__device__ __forceinline__ int mk_nunits(int mode, int c0, int c1) {
  return mode == MODE_GATEUP ? c1 - c0 : (c1 - c0 + 1) >> 1;
}
// Unit u of a staged chunk [c0, c1) (see unit_rows): its two rows.
__device__ __forceinline__ UnitRows mk_unit(const MkPhase& ph, int mode, const uint8_t* stage, int c0, int c1,
                                            const Part (&parts)[3], int u) {
  UnitRows w;
  w.si = 0;
  w.has1 = true;
  if (mode == MODE_QKV) {
    w.r = c0 + 2 * u;
    const int qn = ph.seg[0].rows, kn = ph.seg[1].rows;
    w.si = w.r < qn ? 0 : (w.r < qn + kn ? 1 : 2);
    const int sb = w.si == 0 ? 0 : (w.si == 1 ? qn : qn + kn);
    const uint32_t off = w.si == 0 ? parts[0].off : (w.si == 1 ? parts[1].off : parts[2].off);
    const int lo = w.si == 0 ? parts[0].lo : (w.si == 1 ? parts[1].lo : parts[2].lo);
    const int rb = ph.seg[w.si].row_bytes;
    w.p0 = stage + off + (size_t)(w.r - sb - lo) * rb;
    w.p1 = w.p0 + rb;
    w.ty0 = w.ty1 = ph.seg[w.si].type;
  } else if (mode == MODE_GATEUP) {
    w.r = c0 + u;
    w.p0 = stage + (size_t)u * ph.seg[0].row_bytes;
    w.p1 = stage + parts[1].off + (size_t)u * ph.seg[1].row_bytes;
    w.ty0 = ph.seg[0].type;
    w.ty1 = ph.seg[1].type;
  } else {
    w.r = c0 + 2 * u;
    w.p0 = stage + (size_t)(2 * u) * ph.seg[0].row_bytes;
    w.p1 = w.p0 + ph.seg[0].row_bytes;
    w.has1 = w.r + 1 < c1;
    w.ty0 = w.ty1 = ph.seg[0].type;
  }
  return w;
}
// Both dot products of a unit (row_pair_dots: each row's type dispatched at
// run time; the Q4_K / Q6_K rows of a Q4_K_M model take the first branches).
__device__ __forceinline__ float2 mk_dot2(const UnitRows& w, int nb, const ActQ8& act, int lane) {
  return row_pair_dots(w.ty0, w.p0, w.ty1, w.p1, w.has1, nb, act, lane);
}

// Per-warp state carried from phase to phase: the ring position (stage,
// mbarrier parity) and the head's running argmax.
struct MkRun {
  int s, par;
  float best_v;
  int best_i;
};
__device__ __forceinline__ void mk_advance(MkRun& run, int ns) {
  if (++run.s == ns) {
    run.s = 0;
    run.par ^= 1;
  }
}

// The first one or two ring stages of this CTA's rows in phase ph (the
// stages mk_chunks takes first), waited for before the phase's activation
// build: the producer issued them phases earlier, and the wait and its
// bookkeeping then overlap the wait for the phase's inputs instead of
// following the activation build. Slot 10 / 11 of the trace: the wait's start
// and its mbarrier polls.
__device__ __forceinline__ bool mk_first_stages(const MkParams& p, const MkPhase& ph, int phase, int r0, int r1,
                                                uint64_t* full, const MkRun& run, int cw, int lane) {
  if (r0 >= r1) return true;
  const int c1 = min(r0 + ph.chunk_rows, r1);
  const bool two = ph.kind != PH_QKV && c1 < r1;
  uint32_t iters = 0;
  const bool tr = p.trace && cw == 0 && lane == 0;
  if (tr) mk_stamp(p, phase, 10);
  if (!mk_wait(&full[run.s], (uint32_t)run.par, p.err, tr ? &iters : nullptr)) return false;
  if (tr) p.trace[((size_t)phase * gridDim.x + blockIdx.x) * MK_TRACE_SLOTS + 11] = iters;
  if (two) {
    const bool wrap = run.s + 1 == p.ns;
    if (!mk_wait(&full[wrap ? 0 : run.s + 1], (uint32_t)(run.par ^ (wrap ? 1 : 0)), p.err)) return false;
  }
  return true;
}

// All chunks of this CTA's rows in one matvec phase: wait for the stages,
// compute, hand the stages back to the producer. Except for QKV (few rows
// per CTA), chunks are taken two at a time and their units dealt over the
// consumer warps as one list, so a phase whose rows arrive in several stages
// does not serialise one unit per warp per stage.
// Rows [r0, r1) come from phase_rows; the first chunk's stages were already
// waited for (mk_first_stages) when first_waited is set.
__device__ MkRun mk_chunks(const MkParams& p, const MkPhase& ph, int mode, int phase, int pos, uint32_t tag,
                           uint8_t* smem, uint64_t* full, uint64_t* empty, MkRun run, const ActQ8 act, int cw,
                           int lane, int r0, int r1, bool first_waited) {
  const MkCtx cx{p, ph, pos, phase, tag};
  const int nb = ph.nb;
  for (int c0 = r0; c0 < r1;) {
    const int c1 = min(c0 + ph.chunk_rows, r1);
    const bool two = mode != MODE_QKV && c1 < r1;
    const int c2 = two ? min(c1 + ph.chunk_rows, r1) : c1;
    const int sA = run.s, pA = run.par;
    mk_advance(run, p.ns);
    const int sB = run.s, pB = run.par;
    if (two) mk_advance(run, p.ns);
    if (!(first_waited && c0 == r0)) {
      if (!mk_wait(&full[sA], (uint32_t)pA, p.err)) return run;
      if (two && !mk_wait(&full[sB], (uint32_t)pB, p.err)) return run;
    }
    if (c0 == r0 && cw == 0 && lane == 0) mk_stamp(p, phase, 4);
    Part pa[3], pb[3];
    mk_parts(ph, mode, c0, c1, pa);
    if (two) mk_parts(ph, mode, c1, c2, pb);
    const int nA = mk_nunits(mode, c0, c1), U = nA + (two ? mk_nunits(mode, c1, c2) : 0);
    const uint8_t* stA = smem + (size_t)sA * MK_STAGE;
    const uint8_t* stB = smem + (size_t)sB * MK_STAGE;
    for (int g = cw; g < U; g += MK_CW) {
      const bool inA = g < nA;
      Part q[3];
#pragma unroll
      for (int k = 0; k < 3; k++) q[k] = inA ? pa[k] : pb[k];
      const UnitRows w = mk_unit(ph, mode, inA ? stA : stB, inA ? c0 : c1, inA ? c1 : c2, q, inA ? g : g - nA);
      float cs = 0.f, sn = 0.f;
      if (mode == MODE_QKV && w.si < 2) {  // RoPE factors, loaded before the dots
        const int hd = p.hd, rr = w.si == 0 ? w.r : w.r - ph.seg[0].rows;
        const size_t ti = (size_t)pos * (hd >> 1) + ((rr % hd) >> 1);
        cs = __ldg(p.cos_t + ti);
        sn = __ldg(p.sin_t + ti);
      }
      const float2 d = mk_dot2(w, nb, act, lane);
      if (lane == 0) {
        if (mode == MODE_QKV) unit_epilogue<MODE_QKV>(cx, w, d.x, d.y, cs, sn, run.best_v, run.best_i);
        else if (mode == MODE_GATEUP) unit_epilogue<MODE_GATEUP>(cx, w, d.x, d.y, cs, sn, run.best_v, run.best_i);
        else if (mode == MODE_HEAD) unit_epilogue<MODE_HEAD>(cx, w, d.x, d.y, cs, sn, run.best_v, run.best_i);
        else unit_epilogue<MODE_RESID>(cx, w, d.x, d.y, cs, sn, run.best_v, run.best_i);
      }
    }
    __syncwarp();
    if (c0 == r0 && cw == 0 && lane == 0) mk_stamp(p, phase, 5);
    if (lane == 0) {
      mbar_arrive(&empty[sA]);
      if (two) mbar_arrive(&empty[sB]);
    }
    c0 = c2;
  }
  return run;
}

template <typename KV>
__device__ __forceinline__ float4 kv_load4(const KV* base, size_t idx) {
  if constexpr (sizeof(KV) == 4) {
    return __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx));
  } else {
    const uint2 r = __ldcg(reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(base) + idx));
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
}

// ---------------------------------------------------------------------------
// Consumer: attention unit (g, s) = kv head g, context split s of `splits`,
// on all consumer warps. Tiles of MK_ATT_TILE(HD) positions: K and V of the
// tile are staged in shared memory with one wave of loads, then scores
// (thread per (head, position)), online softmax (warp per head) and P.V
// (thread per (head, dimension)). With splits > 1 the split partials go
// through global memory and the last split's CTA merges them. q and this
// step's K/V row are the QKV phase's tagged words (tag `want`; earlier
// positions come from the cache, written by earlier steps); y is written as
// tagged words (tag `tag`).
// ---------------------------------------------------------------------------
template <int HD>
constexpr int mk_att_tile() { return 4096 / HD; }

// Shared-memory floats of the attention unit.
__host__ __device__ inline size_t mk_att_floats(int hd, int nrep) {
  const int tile = 4096 / hd;
  return (size_t)nrep * hd + (size_t)tile * (hd + 1) + (size_t)tile * hd + (size_t)nrep * tile +
         3 * (size_t)nrep + 2 * (size_t)ATT_SPLITS * nrep + nrep + 1;
}

template <int HD, typename KV>
__device__ void mk_attn_unit(const MkParams& p, const MkPhase& ph, int g, int r0, int nh, int s, int splits,
                             int T, float* sm, int cw, int lane, uint32_t want, uint32_t tag) {
  constexpr int TILE = mk_att_tile<HD>();
  constexpr int MAXE = (ATT_MAX_REP * HD + MK_CT - 1) / MK_CT;  // (head, dim) elements per thread
  const int nrep = p.n_head / p.n_kv;   // heads of group g; this unit takes [r0, r0 + nh)
  const int tid = cw * 32 + lane;
  float* qs = sm;                              // [nrep][HD]
  float* Ks = qs + nrep * HD;                  // [TILE][HD + 1]
  float* Vs = Ks + TILE * (HD + 1);            // [TILE][HD]
  float* ps = Vs + TILE * HD;                  // [nrep][TILE]
  float* mrow = ps + nrep * TILE;              // [nrep]
  float* lrow = mrow + nrep;
  float* corr = lrow + nrep;
  float* cw_m = corr + nrep;                   // [ATT_SPLITS][nrep]
  float* cw_l = cw_m + ATT_SPLITS * nrep;
  float* ltot = cw_l + ATT_SPLITS * nrep;      // [nrep]
  int* s_last = reinterpret_cast<int*>(ltot + nrep);

  const int chunk = (T + splits - 1) / splits;
  const int t0 = min(T, s * chunk), t1 = min(T, t0 + chunk);
  const int64_t kvbase = (int64_t)g * p.max_seq * HD;
  const KV* kc = reinterpret_cast<const KV*>(ph.kc) + kvbase;
  const KV* vc = reinterpret_cast<const KV*>(ph.vc) + kvbase;
  const unsigned long long* qw = p.fq + (size_t)(g * nrep + r0) * HD;
  for (int i = tid; i < nh * HD; i += MK_CT) qs[i] = wait_word<false>(qw + i, want, p.err, p.poll_limit);
  if (tid < nh) { mrow[tid] = -INFINITY; lrow[tid] = 0.f; }
  float o[MAXE];
#pragma unroll
  for (int k = 0; k < MAXE; k++) o[k] = 0.f;
  constexpr int V4 = HD / 4;
  for (int tb = t0; tb < t1; tb += TILE) {
    const int n = min(TILE, t1 - tb);
    for (int i = tid; i < n * V4; i += MK_CT) {
      const int tt = i / V4, c = (i % V4) * 4;
      float4 kv, vv;
      if (tb + tt == T - 1) {  // this step's row
        unsigned long long kw[4], vw[4];
                wait_words<false, 4>(p.fkv + (size_t)g * HD + c, want, kw, p.err, p.poll_limit);
        wait_words<false, 4>(p.fkv + ((size_t)p.n_kv + g) * HD + c, want, vw, p.err, p.poll_limit);
        kv = make_float4(word_val(kw[0]), word_val(kw[1]), word_val(kw[2]), word_val(kw[3]));
        vv = make_float4(word_val(vw[0]), word_val(vw[1]), word_val(vw[2]), word_val(vw[3]));
      } else {
        kv = kv_load4(kc, (size_t)(tb + tt) * HD + c);
        vv = kv_load4(vc, (size_t)(tb + tt) * HD + c);
      }
      float* kd = Ks + tt * (HD + 1) + c;
      kd[0] = kv.x; kd[1] = kv.y; kd[2] = kv.z; kd[3] = kv.w;
      *reinterpret_cast<float4*>(Vs + tt * HD + c) = vv;
    }
    named_sync(1, MK_CT);
    // scores: thread per (head, position)
    for (int e = tid; e < nh * TILE; e += MK_CT) {
      const int h = e / TILE, t = e % TILE;
      float sc = -INFINITY;
      if (t < n) {
        const float* q = qs + h * HD;
        const float* k = Ks + t * (HD + 1);
        float acc = 0.f;
#pragma unroll 16
        for (int d = 0; d < HD; d++) acc += q[d] * k[d];
        sc = acc * p.att_scale;
      }
      ps[h * TILE + t] = sc;
    }
    named_sync(1, MK_CT);
    // online softmax: warp per head
    for (int h = cw; h < nh; h += MK_CW) {
      float mt = -INFINITY;
      for (int t = lane; t < n; t += 32) mt = fmaxf(mt, ps[h * TILE + t]);
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float mold = mrow[h];
      const float mnew = fmaxf(mold, mt);
      float ls = 0.f;
      for (int t = lane; t < TILE; t += 32) {
        const float pe = t < n ? expf(ps[h * TILE + t] - mnew) : 0.f;
        ps[h * TILE + t] = pe;
        ls += pe;
      }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
      if (lane == 0) {
        const float c = expf(mold - mnew);  // 0 on the first tile (mold = -inf)
        corr[h] = c;
        lrow[h] = lrow[h] * c + ls;
        mrow[h] = mnew;
      }
    }
    named_sync(1, MK_CT);
    // P.V: thread per (head, dimension)
#pragma unroll
    for (int k = 0; k < MAXE; k++) {
      const int e = tid + k * MK_CT;
      if (e < nh * HD) {
        const int h = e / HD, d = e % HD;
        float acc = o[k] * corr[h];
        const float* pr = ps + h * TILE;
        for (int t = 0; t < n; t++) acc += pr[t] * Vs[t * HD + d];
        o[k] = acc;
      }
    }
    named_sync(1, MK_CT);
  }
  const int y0 = (g * nrep + r0) * HD;  // this unit's rows of y
  if (splits == 1) {
#pragma unroll
    for (int k = 0; k < MAXE; k++) {
      const int e = tid + k * MK_CT;
      if (e < nh * HD) st_word_gpu(p.fy + y0 + e, tag_word(tag, o[k] / lrow[e / HD]));
    }
    return;
  }
  const size_t pbase = (((size_t)g * ATT_SPLITS + s) * nrep + r0) * (HD + 2);
#pragma unroll
  for (int k = 0; k < MAXE; k++) {
    const int e = tid + k * MK_CT;
    if (e < nh * HD) p.att_part[pbase + (size_t)(e / HD) * (HD + 2) + e % HD] = o[k];
  }
  if (tid < nh) {
    p.att_part[pbase + (size_t)tid * (HD + 2) + HD] = mrow[tid];
    p.att_part[pbase + (size_t)tid * (HD + 2) + HD + 1] = lrow[tid];
  }
  __threadfence();
  named_sync(1, MK_CT);
  if (tid == 0) {
    const unsigned prev = atomicAdd(&p.att_cnt[g * nrep + r0], 1u);
    *s_last = (prev == (unsigned)splits - 1);
  }
  named_sync(1, MK_CT);
  if (!*s_last) return;
  __threadfence();
  // the last split of head g merges all splits
  const size_t base0 = ((size_t)g * ATT_SPLITS) * nrep * (HD + 2);
  for (int i = tid; i < splits * nh; i += MK_CT) {
    const int s2 = i / nh, h = i % nh;
    const size_t o2 = base0 + ((size_t)s2 * nrep + r0 + h) * (HD + 2);
    cw_m[s2 * nh + h] = __ldcg(p.att_part + o2 + HD);
    cw_l[s2 * nh + h] = __ldcg(p.att_part + o2 + HD + 1);
  }
  named_sync(1, MK_CT);
  if (tid < nh) {
    float M = -INFINITY;
    for (int s2 = 0; s2 < splits; s2++)
      if (cw_l[s2 * nh + tid] > 0.f) M = fmaxf(M, cw_m[s2 * nh + tid]);
    float Ls = 0.f;
    for (int s2 = 0; s2 < splits; s2++) {
      const float lv = cw_l[s2 * nh + tid];
      const float w = lv > 0.f ? expf(cw_m[s2 * nh + tid] - M) : 0.f;
      cw_m[s2 * nh + tid] = w;
      Ls += lv * w;
    }
    ltot[tid] = Ls;
  }
  named_sync(1, MK_CT);
  for (int e = tid; e < nh * HD; e += MK_CT) {
    const int h = e / HD, d = e % HD;
    float O = 0.f;
    for (int s2 = 0; s2 < splits; s2++) {
      const float w = cw_m[s2 * nh + h];
      if (w != 0.f) O += w * __ldcg(p.att_part + base0 + ((size_t)s2 * nrep + r0 + h) * (HD + 2) + d);
    }
    st_word_gpu(p.fy + ((size_t)g * nrep + r0 + h) * HD + d, tag_word(tag, O / ltot[h]));
  }
  if (tid == 0) p.att_cnt[g * nrep + r0] = 0u;
}

// ---------------------------------------------------------------------------
// Consumer: short-context attention, one unit per query head hq, no tiles or
// splits (T <= MK_ATT_SHORT_PASSES * positions per pass). Thread (pi, di)
// holds dims [8 di, 8 di + 8) of positions pi, pi + P, ... (P = positions per
// pass): the K rows of the cache are loaded into registers before the unit
// waits for q, each score is a dot over 8 dims reduced across the HD / 8
// threads of its position, softmax max and sum are block reductions, and the
// V rows are loaded while those run. P.V partials are reduced across the
// positions of a warp by shuffles, then across warps in shared memory.
// ---------------------------------------------------------------------------
constexpr int MK_ATT_SHORT_PASSES = 4;
template <int HD>
__host__ __device__ constexpr int mk_att_short_max_t() { return MK_ATT_SHORT_PASSES * (MK_CT / (HD / 8)); }

template <typename KV>
__device__ __forceinline__ void kv_load8(const KV* base, size_t idx, float (&v)[8]) {
  if constexpr (sizeof(KV) == 4) {
    const float4* s = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx);
    const float4 a = __ldcg(s), b = __ldcg(s + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 r = __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(base) + idx));
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

template <int HD, typename KV>
__device__ void mk_attn_short(const MkParams& p, const MkPhase& ph, int phase, int hq, int T, float* sm, int cw,
                              int lane, uint32_t want, uint32_t tag) {
  constexpr int TPP = HD / 8;       // threads per position
  constexpr int PPP = MK_CT / TPP;  // positions per pass
  constexpr int NP = MK_ATT_SHORT_PASSES;
  const int tid = cw * 32 + lane, pi = tid / TPP, di = tid % TPP;
  const int g = hq / (p.n_head / p.n_kv);
  const int64_t kvbase = (int64_t)g * p.max_seq * HD;
  const KV* kc = reinterpret_cast<const KV*>(ph.kc) + kvbase;
  const KV* vc = reinterpret_cast<const KV*>(ph.vc) + kvbase;
  float* red = sm;               // [2][MK_CW] warp maxima / sums
  float* opart = sm + 2 * MK_CW; // [MK_CW][HD] P.V partials
  // K rows written by earlier steps: loads issued before q is awaited
  float kr[NP][8];
#pragma unroll
  for (int k = 0; k < NP; k++) {
    const int t = pi + k * PPP;
    if (t < T - 1) kv_load8(kc, (size_t)t * HD + 8 * di, kr[k]);
  }
  if (tid == 0) mk_stamp(p, phase, 3);
  float q[8];
  {
    unsigned long long w[8];
    wait_words<false, 8>(p.fq + (size_t)hq * HD + 8 * di, want, w, p.err, p.poll_limit);
#pragma unroll
    for (int e = 0; e < 8; e++) q[e] = word_val(w[e]);
  }
  if (tid == 0) mk_stamp(p, phase, 4);
  const int tl = T - 1;  // this step's K/V row, from the QKV phase
  if (tl % PPP == pi) {
    unsigned long long w[8];
    wait_words<false, 8>(p.fkv + (size_t)g * HD + 8 * di, want, w, p.err, p.poll_limit);
#pragma unroll
    for (int k = 0; k < NP; k++)
      if (k == tl / PPP) {
#pragma unroll
        for (int e = 0; e < 8; e++) kr[k][e] = word_val(w[e]);
      }
  }
  float sc[NP];
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < NP; k++) {
    float a = 0.f;
#pragma unroll
    for (int e = 0; e < 8; e++) a += q[e] * kr[k][e];
#pragma unroll
    for (int off = TPP / 2; off >= 1; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
    sc[k] = pi + k * PPP < T ? a * p.att_scale : -INFINITY;
    mx = fmaxf(mx, sc[k]);
  }
  if (tid == 0) mk_stamp(p, phase, 5);
  // V rows: loads issued before the softmax reductions
  float vr[NP][8];
#pragma unroll
  for (int k = 0; k < NP; k++) {
    const int t = pi + k * PPP;
    if (t < T - 1) kv_load8(vc, (size_t)t * HD + 8 * di, vr[k]);
  }
  if (tl % PPP == pi) {
    unsigned long long w[8];
    wait_words<false, 8>(p.fkv + ((size_t)p.n_kv + g) * HD + 8 * di, want, w, p.err, p.poll_limit);
#pragma unroll
    for (int k = 0; k < NP; k++)
      if (k == tl / PPP) {
#pragma unroll
        for (int e = 0; e < 8; e++) vr[k][e] = word_val(w[e]);
      }
  }
#pragma unroll
  for (int off = 16; off >= TPP; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if (lane == 0) red[cw] = mx;
  named_sync(1, MK_CT);
  float M = red[0];
  for (int w = 1; w < MK_CW; w++) M = fmaxf(M, red[w]);
  if (tid == 0) mk_stamp(p, phase, 6);
  float l = 0.f, o[8];
#pragma unroll
  for (int e = 0; e < 8; e++) o[e] = 0.f;
#pragma unroll
  for (int k = 0; k < NP; k++) {
    if (pi + k * PPP < T) {
      const float pe = expf(sc[k] - M);
      l += pe;
#pragma unroll
      for (int e = 0; e < 8; e++) o[e] += pe * vr[k][e];
    }
  }
  // each position's weight is held by all TPP threads of it: count it once
#pragma unroll
  for (int off = 16; off >= TPP; off >>= 1) {
    l += __shfl_xor_sync(0xffffffffu, l, off);
#pragma unroll
    for (int e = 0; e < 8; e++) o[e] += __shfl_xor_sync(0xffffffffu, o[e], off);
  }
  if (lane == 0) red[MK_CW + cw] = l;
  if (lane < TPP) {
#pragma unroll
    for (int e = 0; e < 8; e++) opart[cw * HD + 8 * lane + e] = o[e];
  }
  named_sync(1, MK_CT);
  if (tid == 0) mk_stamp(p, phase, 7);
  if (tid < HD) {
    float L = 0.f, O = 0.f;
    for (int w = 0; w < MK_CW; w++) {
      L += red[MK_CW + w];
      O += opart[w * HD + tid];
    }
    st_word_gpu(p.fy + (size_t)hq * HD + tid, tag_word(tag, O / L));
  }
  named_sync(1, MK_CT);
  if (tid == 0) mk_stamp(p, phase, 8);
}

// Asynchronous copy of a phase descriptor into shared memory by one warp
// (8-byte pieces); the warp waits for it (cp.async.wait_all) before the sync
// that publishes it.
__device__ __forceinline__ void mk_fetch_phase(const MkPhase* src, MkPhase* dst, int lane) {
  static_assert(sizeof(MkPhase) % 8 == 0, "phase descriptor copied in 8-byte pieces");
  constexpr int W8 = (int)(sizeof(MkPhase) / 8);
  for (int w = lane; w < W8; w += 32)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(reinterpret_cast<uint64_t*>(dst) + w)),
                 "l"(reinterpret_cast<const uint64_t*>(src) + w)
                 : "memory");
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <int HD, typename KV>
__global__ void __launch_bounds__(MK_THREADS, 1) k_decode_mega(const __grid_constant__ MkParams params) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_flag;
  __shared__ __align__(16) MkPhase s_ph[3];  // phase i's descriptor in s_ph[i % 3]
  __shared__ int s_pos;  // position of this step's token (constant during the step)
  // The launch parameters live in shared memory for the whole step: read
  // through the constant cache, which shares its backing store with the
  // instruction cache, they missed again and again.
  __shared__ __align__(16) MkParams p;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(&params);
    uint32_t* dst = reinterpret_cast<uint32_t*>(&p);
    for (int w = tid; w < (int)(sizeof(MkParams) / 4); w += blockDim.x) dst[w] = src[w];
  }
  __syncthreads();
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bars);
  uint64_t* empty = full + MK_MAX_NS;
  if (tid == 0) {
    mk_stamp(p, p.n_ph, 0);  // kernel entry
    for (int s = 0; s < p.ns; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], MK_CW);
    }
    mbar_init(empty + MK_MAX_NS, 1);  // rmsnorm weights staged in the attention region
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) mk_producer(p, smem);
    return;
  }
  const int ctid = tid - 32, cw = warp - 1;
  if (ctid == 0) s_pos = (int)__ldcg(p.pos);
  float* xrep = reinterpret_cast<float*>(smem + p.off_xrep);
  const ActQ8 act{reinterpret_cast<int8_t*>(smem + p.off_act_qs), reinterpret_cast<float*>(smem + p.off_act_d),
                  reinterpret_cast<int32_t*>(smem + p.off_act_bs), reinterpret_cast<int8_t*>(smem + p.off_act0_qs),
                  reinterpret_cast<float*>(smem + p.off_act0_d), reinterpret_cast<int32_t*>(smem + p.off_act0_s)};
  MkRun run{0, 0, -INFINITY, 0x7fffffff};
  uint64_t* gbar = empty + MK_MAX_NS;
  uint32_t gcount = 0;   // gamma stagings consumed so far (mbarrier parity)
  uint32_t gissued = 0;  // gamma stagings issued (consumer thread 0)
  // phase i's outputs carry tag gen + i + 1; its inputs gen + i
  const uint32_t gen = (uint32_t)(__ldcg(p.epoch) * (unsigned long long)(p.n_ph + 1));

  // Phase descriptors live in shared memory, three deep: phases 0 and 1 are
  // copied here; phase i + 2's is fetched asynchronously at the start of
  // phase i (into the buffer of phase i - 1, which no warp reads once all
  // passed phase i's start), so no phase start waits for a global load.
  for (int i = 0; i < 2 && i < p.n_ph; i++) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(p.ph + i);
    uint32_t* dst = reinterpret_cast<uint32_t*>(&s_ph[i]);
    for (int w = ctid; w < (int)(sizeof(MkPhase) / 4); w += MK_CT) dst[w] = __ldg(src + w);
  }
  // The device error word as loaded at the previous phase start (consumer
  // thread 0): checked one phase late, so its load never stalls a phase
  // start. Every wait inside a phase checks the word itself.
  uint32_t err_seen = 0u;

  for (int i = 0; i < p.n_ph; i++) {
    // the sync below also ends the CTA's previous phase, so the attention
    // region is free for the rmsnorm weights staged next
    MkPhase& ph = s_ph[i % 3];
    if (cw == 0) asm volatile("cp.async.wait_all;" ::: "memory");  // phase i + 1's descriptor
    if (ctid == 0) s_flag = err_seen != 0u;
    named_sync(1, MK_CT);
    if (s_flag) {  // a wait gave up somewhere: all consumer warps leave together
      if (ctid == 0 && gissued > gcount) mk_drain(gbar, (gissued - 1u) & 1u);  // no copy left in flight
      return;
    }
    if (ctid == 0) err_seen = *reinterpret_cast<const volatile uint32_t*>(p.err);
    if (cw == 0 && i + 2 < p.n_ph) mk_fetch_phase(p.ph + i + 2, &s_ph[(i + 2) % 3], lane);
    // Stage the rmsnorm weights of the next phase (gate/up after attn_output,
    // q/k/v or the head after ffn_down; phase 0 its own) in the attention
    // region, idle until then, so the prologue reads them from shared memory.
    if (ctid == 0) {
      const int gi = i == 0 ? 0 : ((ph.kind == PH_WO || ph.kind == PH_DOWN) && i + 1 < p.n_ph ? i + 1 : -1);
      const float* g = gi < 0 ? nullptr : s_ph[gi % 3].gamma;  // phase gi's descriptor is in place
      if (g) {
        const uint32_t bytes = (uint32_t)s_ph[gi % 3].K * 4u;
        fence_proxy_async();
        mbar_expect_tx(gbar, bytes);
        bulk_g2s(smem + p.off_att, g, bytes, gbar, l2_evict_first_policy());
        gissued++;
      }
    }
    if (ctid == 0) mk_stamp(p, i, 0);
    const uint32_t want = gen + (uint32_t)i, tag = want + 1u;
    if (ph.kind == PH_ATTN) {
      // Split the context across CTAs only when it spans several tiles.
      const int T = s_pos + 1;
      constexpr int per = 2 * mk_att_tile<HD>();
      const int splits = min(ATT_SPLITS, (T + per - 1) / per);
      // Short contexts: one unit per query head (more CTAs, the K/V tile is
      // re-read from L2 by each head of a group); long contexts: one unit per
      // KV head (every K/V byte read once).
      const int nrep = p.n_head / p.n_kv;
      const int hpu = T <= MK_ATT_PER_HEAD_MAX_T ? 1 : nrep, hsplit = nrep / hpu;
      const int nunits = p.n_kv * hsplit * splits;
      float* asm_ = reinterpret_cast<float*>(smem + p.off_att);
      if (T <= mk_att_short_max_t<HD>()) {
        // one unit per query head, spread over the grid
        for (int u = blockIdx.x; u < p.n_head; u += gridDim.x)
          mk_attn_short<HD, KV>(p, ph, i, u, T, asm_, cw, lane, want, tag);
      } else
      for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
        const int hu = u / splits;  // head unit: (KV head, first query head of the unit)
        mk_attn_unit<HD, KV>(p, ph, hu / hsplit, (hu % hsplit) * hpu, hpu, u % splits, splits, T, asm_, cw, lane,
                             want, tag);
      }
    } else {
      int r0, r1;
      phase_rows(ph, r0, r1);
      const bool staged = mk_first_stages(p, ph, i, r0, r1, full, run, cw, lane);
      mk_build_act(p, ph, i, smem, act, cw, lane, xrep, gbar, gcount & 1u, want);
      if (ph.gamma) gcount++;
      if (ctid == 0) mk_stamp(p, i, 1);
      // a wait that gives up flags the error and goes on (in bounds); all
      // warps leave at the next phase start
      const int mode = mode_of(ph.kind);
      if (staged) run = mk_chunks(p, ph, mode, i, s_pos, tag, smem, full, empty, run, act, cw, lane, r0, r1, true);
    }
    if (ctid == 0) mk_stamp(p, i, 2);
  }
  // HEAD: CTA argmax partial, the last CTA reduces all partials.
  float* rv = reinterpret_cast<float*>(smem + p.off_red);
  int* ri = reinterpret_cast<int*>(rv + 32);
  if (lane == 0) { rv[cw] = run.best_v; ri[cw] = run.best_i; }
  named_sync(1, MK_CT);
  if (ctid == 0) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int w = 0; w < MK_CW; w++)
      if (am_better(rv[w], ri[w], bv, bi)) { bv = rv[w]; bi = ri[w]; }
    p.am_val[blockIdx.x] = bv;
    p.am_idx[blockIdx.x] = bi;
    __threadfence();
    const unsigned prev = atomicAdd(p.am_cnt, 1u);
    s_flag = (prev == gridDim.x - 1);
  }
  named_sync(1, MK_CT);
  if (!s_flag) return;
  __threadfence();
  if (cw == 0) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = lane; i < (int)gridDim.x; i += 32) {
      const float v = __ldcg(p.am_val + i);
      const int ix = __ldcg(p.am_idx + i);
      if (am_better(v, ix, bv, bi)) { bv = v; bi = ix; }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (am_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    const unsigned long long ep = __ldcg(p.epoch);
    if (lane == 0 && p.tp > 1) {
      // every rank's winner (value, global row) to every rank, then the
      // reference's order: larger value, then smaller row; NaN never wins
      const size_t base = (size_t)(ep & 1) * p.tp * 2;
      for (int k = 0; k < p.tp; k++) {
        uint32_t* hs = p.hslot[k] + base + (size_t)p.tp_rank * 2;
        hs[0] = __float_as_uint(bv);
        hs[1] = bi == 0x7fffffff ? 0xffffffffu : (uint32_t)(bi + p.v0);
      }
      for (int k = 0; k < p.tp; k++) red_release_sys_add64(p.hctr[k], 1ull);
      float gv = -INFINITY;
      uint32_t gi = 0xffffffffu;
      if (wait_ge_sys(p.hctr[p.tp_rank], (ep + 1) * (unsigned long long)p.tp, p.err)) {
        const uint32_t* hs = p.hslot[p.tp_rank] + base;
        for (int r = 0; r < p.tp; r++) {
          const float v = __uint_as_float(hs[2 * r]);
          const uint32_t ix = hs[2 * r + 1];
          if (ix != 0xffffffffu && (gi == 0xffffffffu || v > gv || (v == gv && ix < gi))) { gv = v; gi = ix; }
        }
      }
      bi = gi == 0xffffffffu ? 0x7fffffff : (int)gi;
    }
    if (lane == 0) {
      *p.token = (bi == 0x7fffffff) ? 0u : (uint32_t)bi;
      *p.pos = __ldcg(p.pos) + 1;
      *p.am_cnt = 0u;
      // every CTA has read the epoch (it reached am_cnt after the head
      // phase): the next step's tags start after this step's
      *p.epoch = ep + 1;
      mk_stamp(p, p.n_ph, 1);  // step result written
    }
  }
}

}  // namespace armai
