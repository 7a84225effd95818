// sm_100a kernels and the C ABI of the KG constraint engine.
//
// Per decoding step the serving path runs one kernel, sync_apply_kernel: a CTA per request
// row whose warp 0 applies the row's admission, consumes its new tokens and rebuilds its
// allowed-token bitmask (core.cuh), after which all eight warps write -inf over the row's
// disallowed columns.  The separate entry points run the same pieces apart: step_kernel
// (one warp per row: advance or sync, mask rebuilt where the state changes) and
// apply_kernel (a flat grid over row chunks writing -inf, HBM-write bound); draft rows and
// the logit policies (release, escape bias), which need a whole row per CTA, use
// draft_apply_kernel.  The reference runs a step as sync_kernel + row_mask_kernel +
// [escape_bias_kernel] + [release_kernel] + apply_kernel (csrc/engine.cu:2057-2074,
// 2372-2587).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "core.cuh"

namespace xg {

constexpr int32_t kWarpsPerBlock = 1;  // one row per CTA: rows spread over every SM
constexpr int32_t kApplyThreads = 256;
constexpr int32_t kApplyBatch = 4;        // 1024-column segments whose loads a warp issues together
constexpr int32_t kApplyCtasPerSm = 4;    // apply grid: CTAs per SM the row split aims at
constexpr int32_t kFusedThreads = 256;    // sync_apply: warp 0 advances, all 8 warps write
constexpr int32_t kFusedRegisters = 128;  // sync_apply: room for a whole state in registers (2 CTAs/SM)
constexpr int32_t kDelimCopy = 1024;      // sync_apply: delimiter start tokens copied to shared memory

struct __align__(16) WarpShared {
  Key top[kTopCap];
  int32_t scratch[kScratchInts + 2];
};

__device__ __forceinline__ Ctx make_ctx(const Tables& t, int32_t slot, WarpShared& sh) {
  return Ctx{t, Warp{static_cast<int32_t>(threadIdx.x & 31)}, slot,
             t.memory + static_cast<int64_t>(slot) * t.memory_ints, sh.top, sh.scratch};
}

// A slot's state into every lane of the warp: lane k loads words k and k + 32 (two
// coalesced loads), then each word is broadcast by a shuffle (every lane holds the whole
// state, in registers).
__device__ __forceinline__ XgState load_state(const Tables& t, int32_t slot) {
  static_assert(sizeof(XgState) == 64 * sizeof(int32_t), "XgState is 64 words");
  const int32_t lane = threadIdx.x & 31;
  const int32_t* from = reinterpret_cast<const int32_t*>(t.states + slot);
  const int32_t lo = from[lane], hi = from[lane + 32];
  union {
    XgState s;
    int32_t w[64];
  } u;
#pragma unroll
  for (int32_t k = 0; k < 32; ++k) {
    u.w[k] = __shfl_sync(0xffffffffu, lo, k);
    u.w[k + 32] = __shfl_sync(0xffffffffu, hi, k);
  }
  return u.s;
}

// Every lane holds the same state: lane k stores words k and k + 32 (two coalesced stores
// instead of one lane storing all 64 words).
__device__ __forceinline__ void store_state(const Tables& t, int32_t slot, const XgState& s) {
  static_assert(sizeof(XgState) == 64 * sizeof(int32_t), "XgState is 64 words");
  const int32_t lane = threadIdx.x & 31;
  const int32_t* from = reinterpret_cast<const int32_t*>(&s);
  int32_t* to = reinterpret_cast<int32_t*>(t.states + slot);
  to[lane] = from[lane];
  to[lane + 32] = from[lane + 32];
  __syncwarp();
}

struct StepArgs {
  const int32_t* slots;      // sync: slot per entry; advance: null (entry i is slot i)
  const int32_t* tokens;     // advance: one token per entry
  const int32_t* history;    // sync: [slots, stride]
  int64_t stride;
  const int32_t* prompt_len;
  const int32_t* total_len;
  int32_t count;
};

// Advance (tokens) or sync (history) one slot per warp, then rebuild its mask.
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    step_kernel(const __grid_constant__ Tables t, const StepArgs a) {
  __shared__ WarpShared shared[kWarpsPerBlock];
  // Let a dependent apply_kernel launch now; it waits (griddepcontrol.wait) for this
  // grid to complete and flush before it reads any mask.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int32_t warp = threadIdx.x >> 5;
  const int32_t i = blockIdx.x * kWarpsPerBlock + warp;
  if (i >= a.count) return;  // warp-uniform
  const int32_t slot = a.slots ? a.slots[i] : i;
  Ctx c = make_ctx(t, slot, shared[warp]);
  XgState s = t.states[slot];
  if (a.history) {
    if (!t.active[slot]) return;
    int32_t cursor = t.cursors[slot] < 0 ? a.prompt_len[slot] : t.cursors[slot];
    const int32_t end = a.total_len[slot];
    if (cursor >= end) {
      if ((threadIdx.x & 31) == 0) t.cursors[slot] = cursor;
      return;
    }
    const int32_t* tokens = a.history + a.stride * slot;
    for (; cursor < end; ++cursor) {
      const int32_t token = tokens[cursor];  // in flight while the state's reads are started
      if (s.phase == kSpan) prefetch_span(c, s);
      advance_state(c, s, token);
    }
    if ((threadIdx.x & 31) == 0) t.cursors[slot] = cursor;
  } else {
    const int32_t token = a.tokens[i];
    if (s.phase == kSpan) prefetch_span(c, s);
    advance_state(c, s, token);
  }
  store_state(t, slot, s);
  build_mask(c, s);
}

// Lifecycle of one slot, one warp: 0 open a span, 1 select a version, 2 anchor rows.
struct SlotArgs {
  int32_t slot, op, value, count;
  int32_t rows[kMaxSet];
};

__global__ void __launch_bounds__(32) slot_kernel(const __grid_constant__ Tables t, const SlotArgs a) {
  __shared__ WarpShared shared[1];
  Ctx c = make_ctx(t, a.slot, shared[0]);
  XgState s = t.states[a.slot];
  if (a.op == 0) {
    if (s.phase != kError) {
      s.answer_complete = 0;
      open_span(c, s);
    }
  } else if (a.op == 1) {
    if (c.w.leader()) {
      c.mem[kMemVersion] = a.value;
      c.mem[kMemPendingLo] = -1;
    }
    __syncwarp();
    if (s.phase == kSpan) set_flags(c, s);  // a KG read changed under the open span
  } else {
    if (threadIdx.x < a.count) c.mem[kMemReachedRows + threadIdx.x] = a.rows[threadIdx.x];
    if (threadIdx.x + 32 < a.count) c.mem[kMemReachedRows + threadIdx.x + 32] = a.rows[threadIdx.x + 32];
    if (c.w.leader()) {
      c.mem[kMemReached] = a.count;
      c.mem[kMemPendingLo] = -1;
    }
    __syncwarp();
    if (s.phase == kSpan) set_flags(c, s);
  }
  store_state(t, a.slot, s);
  build_mask(c, s);
}

// begin/end: listed slots back to the initial state (free text, base KG, no binding).
__global__ void begin_kernel(const __grid_constant__ Tables t, const int32_t* slots, int32_t count,
                             int32_t on, int32_t max_slots) {
  const int32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  const int32_t slot = slots ? slots[i] : i;
  if (slot < 0 || slot >= max_slots) return;
  XgState* s = t.states + slot;
  int32_t* words = reinterpret_cast<int32_t*>(s);
  for (int32_t k = 0; k < XG_STATE_INTS; ++k) words[k] = 0;
  int32_t* mem = t.memory + static_cast<int64_t>(slot) * t.memory_ints;
  mem[kMemFacts] = mem[kMemReached] = mem[kMemFrontier] = mem[kMemVersion] = 0;
  mem[kMemPendingLo] = -1;
  t.cursors[slot] = -1;
  t.active[slot] = on;
  t.base[slot] = t.free_mask;
  t.delta[slot] = nullptr;
  if (t.stop_on) t.stop_on[slot] = 0;  // a new request has no STOP table until set_stop
}

// fill_mask: materialize each slot's current mask (base | delta) into its own buffer row;
// the slot then reads it as its delta alone.
__global__ void fill_kernel(const __grid_constant__ Tables t) {
  const int32_t slot = blockIdx.x;
  uint32_t* own = t.masks + static_cast<int64_t>(slot) * t.words_padded;
  const uint32_t* base = t.base[slot];
  const uint32_t* delta = t.delta[slot];
  for (int32_t i = threadIdx.x; i < t.words_padded; i += blockDim.x)
    own[i] = (base ? base[i] : 0u) | (delta ? delta[i] : 0u);
  __syncthreads();
  if (threadIdx.x == 0 && (base || delta)) {
    t.base[slot] = nullptr;
    t.delta[slot] = own;
  }
}

__device__ __forceinline__ uint32_t mask_word(const uint32_t* base, const uint32_t* delta, int64_t w) {
  return (base ? __ldg(base + w) : 0u) | (delta ? delta[w] : 0u);
}

// Allowed bits of the 8 columns starting at column c (c >= 0): a 64-bit window of words.
__device__ __forceinline__ uint32_t allowed8(const uint32_t* base, const uint32_t* delta, int32_t words, int64_t c) {
  const int64_t w = c >> 5;
  const int32_t sh = static_cast<int32_t>(c & 31);
  uint64_t x = w < words ? mask_word(base, delta, w) : 0u;
  if (sh > 24 && w + 1 < words) x |= static_cast<uint64_t>(mask_word(base, delta, w + 1)) << 32;
  return static_cast<uint32_t>(x >> sh) & 0xffu;
}

__device__ __forceinline__ void store_neg8(char* at, uint32_t blocked, uint32_t neg, int elt) {
  if (blocked == 0xffu) {
    if (elt == 2) {
      const uint32_t v = neg | (neg << 16);
      *reinterpret_cast<uint4*>(at) = make_uint4(v, v, v, v);
    } else {
      *reinterpret_cast<uint4*>(at) = make_uint4(neg, neg, neg, neg);
      *reinterpret_cast<uint4*>(at + 16) = make_uint4(neg, neg, neg, neg);
    }
    return;
  }
  for (int32_t k = 0; k < 8; ++k) {
    if ((blocked >> k) & 1u) {
      if (elt == 2)
        *reinterpret_cast<uint16_t*>(at + 2 * k) = static_cast<uint16_t>(neg);
      else
        *reinterpret_cast<uint32_t*>(at + 4 * k) = neg;
    }
  }
}

#ifndef XG_BULK_STORES
#define XG_BULK_STORES 1
#endif

// A run of -inf elements in shared memory (4 KB: one segment of fp32, two of bf16), the
// source of the bulk stores below.  Filled once per CTA; the proxy fence makes the generic
// writes visible to the asynchronous (TMA) proxy after the next CTA barrier.
constexpr int32_t kBlockedRunWords = 1024;

template <int ELT>
__device__ __forceinline__ void fill_blocked_run(uint32_t* run, uint32_t neg, int32_t first = 0) {
  const uint32_t v = ELT == 2 ? (neg | (neg << 16)) : neg;
  for (int32_t k = static_cast<int32_t>(threadIdx.x) - first; k < kBlockedRunWords; k += blockDim.x - first) run[k] = v;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// One bulk (TMA) copy of `bytes` (a multiple of 16) from shared to global memory, both
// 16-byte aligned; completed by bulk_drain.
__device__ __forceinline__ void bulk_store(void* to, const void* from, uint32_t bytes) {
  const uint32_t source = static_cast<uint32_t>(__cvta_generic_to_shared(from));
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(to), "r"(source), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_drain() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Free-text and escaped rows of the automata that block few tokens (most allow every
// token): the row's entry in Tables::sparse, or null (pointer arithmetic, no loads).
__device__ __forceinline__ const int32_t* sparse_row(const Tables& t, const uint32_t* base) {
  const int64_t stride = t.words_padded;  // (a bit is set only for a row the automaton has)
  if (base >= t.free_mask && base < t.free_mask + 32 * stride) {
    const int64_t at = base - t.free_mask;
    if (at % stride == 0 && ((t.free_sparse >> (at / stride)) & 1u)) return t.sparse + (at / stride) * (1 + kSparseBlocked);
  }
  if (base >= t.esc_mask && base < t.esc_mask + 32 * stride) {
    const int64_t at = base - t.esc_mask;
    if (at % stride == 0 && ((t.esc_sparse >> (at / stride)) & 1u))
      return t.sparse + (32 + at / stride) * (1 + kSparseBlocked);
  }
  return nullptr;
}

// Whole CTA: -inf into a sparse row's listed tokens below `cols` (when listed_here), then
// into columns [c0, c1) past the vocabulary.
template <int ELT>
__device__ __forceinline__ void apply_sparse(const Tables& t, char* out, int32_t cols, const int32_t* list,
                                             uint32_t neg, bool listed_here, int64_t c0, int64_t c1) {
  if (listed_here) {
    const int32_t n = list[0];
    for (int32_t k = threadIdx.x; k < n; k += blockDim.x) {
      const int32_t token = list[1 + k];
      if (token >= cols) continue;
      if (ELT == 2)
        *reinterpret_cast<uint16_t*>(out + 2 * static_cast<int64_t>(token)) = static_cast<uint16_t>(neg);
      else
        *reinterpret_cast<uint32_t*>(out + 4 * static_cast<int64_t>(token)) = neg;
    }
  }
  for (int64_t col = (c0 > t.vocab ? c0 : t.vocab) + threadIdx.x; col < c1; col += blockDim.x) {
    if (ELT == 2)
      *reinterpret_cast<uint16_t*>(out + 2 * col) = static_cast<uint16_t>(neg);
    else
      *reinterpret_cast<uint32_t*>(out + 4 * col) = neg;
  }
}

// -inf into the disallowed columns of segments [s0, s1) (1024 columns each) of one
// logits row whose first element is 16-byte aligned; the calling warps split them.
//
// Each lane loads one mask word (32 columns; base | delta), then for store j = 0..3 lane l
// takes the 8-column group g = 32 j + l, fetching its byte of mask from the lane that
// loaded word g / 4 by shuffle, so each store instruction of the warp writes 512
// contiguous bytes (bf16) while the mask costs one load per 32 columns.  A segment with no
// allowed column (most of a row inside a span) is written instead by one bulk copy of the
// shared -inf run `blocked` (when given), issued by lane 0: one instruction for the
// segment, leaving the SM's load/store pipe to the partial segments.  A warp issues the
// loads of kApplyBatch segments before any of their stores (the stores may alias nothing
// the compiler can prove, so it would not hoist the loads itself).
//
// A segment whose allowed and blocked columns interleave densely (a label-root mask: about
// half the vocabulary allowed, scattered) is written column-contiguously instead: in round
// r lane l takes column 32 r + l, so each predicated element store of the warp lands in
// one 128-byte line (64 bytes of bf16) rather than spreading 2-byte pieces over four; the
// L2 request count, which bounds such a row from one SM, falls fourfold, and no logit is
// read.
constexpr int32_t kDenseShare = 4;  // dense: at least 1/4 of its 8-column groups partly blocked

template <int ELT>
__device__ __forceinline__ void apply_segments(const Tables& t, char* out, int32_t cols, const uint32_t* base,
                                               const uint32_t* delta, uint32_t neg, int32_t s0, int32_t s1,
                                               int32_t warp, int32_t warps, const uint32_t* blocked) {
  const int32_t lane = threadIdx.x & 31;
  const int32_t words = t.words;
  bool issued = false;
  for (int32_t first = s0 + warp; first < s1; first += warps * kApplyBatch) {
    uint32_t word[kApplyBatch];
#pragma unroll
    for (int32_t b = 0; b < kApplyBatch; ++b) {
      const int32_t seg = first + b * warps;
      const int32_t w = seg * 32 + lane;
      word[b] = seg < s1 && w < words ? mask_word(base, delta, w) : 0u;  // past the vocabulary: blocked
    }
#pragma unroll
    for (int32_t b = 0; b < kApplyBatch; ++b) {
      const int32_t seg = first + b * warps;  // warp-uniform
      if (seg >= s1) break;
#if XG_BULK_STORES
      if (blocked && (seg + 1) * 1024 <= cols && __ballot_sync(0xffffffffu, word[b] != 0u) == 0u) {
        if (lane == 0) {
          bulk_store(out + static_cast<int64_t>(seg) * 1024 * ELT, blocked, 1024 * ELT);
          issued = true;
        }
        continue;
      }
#endif
      if ((seg + 1) * 1024 <= cols) {
        int32_t partial = 0;  // this lane's 8-column groups that are neither all allowed nor all blocked
#pragma unroll
        for (int32_t k = 0; k < 4; ++k) {
          const uint32_t byte = (word[b] >> (8 * k)) & 0xffu;
          partial += byte != 0u && byte != 0xffu;
        }
        if (__reduce_add_sync(0xffffffffu, partial) * kDenseShare >= 128) {
          char* at = out + (static_cast<int64_t>(seg) * 1024 + lane) * ELT;
#pragma unroll 4
          for (int32_t r = 0; r < 32; ++r) {
            const uint32_t w = __shfl_sync(0xffffffffu, word[b], r);
            if (!((w >> lane) & 1u)) {
              if (ELT == 2)
                *reinterpret_cast<uint16_t*>(at + 64 * r) = static_cast<uint16_t>(neg);
              else
                *reinterpret_cast<uint32_t*>(at + 128 * r) = neg;
            }
          }
          continue;
        }
      }
#pragma unroll
      for (int32_t j = 0; j < 4; ++j) {
        const int32_t g = 32 * j + lane;
        const uint32_t holder = __shfl_sync(0xffffffffu, word[b], g >> 2);
        const int32_t c = seg * 1024 + 8 * g;
        if (c >= cols) continue;
        uint32_t blocked_bits = ~(holder >> (8 * (g & 3))) & 0xffu;
        const int32_t left = cols - c;
        if (left < 8) blocked_bits &= (1u << left) - 1u;
        if (blocked_bits) store_neg8(out + static_cast<int64_t>(c) * ELT, blocked_bits, neg, ELT);
      }
    }
  }
  if (issued) bulk_drain();
}

// Columns [c0, c1) of a row whose start is not 16-byte aligned, one element per thread.
template <int ELT>
__device__ __forceinline__ void apply_scalar(const Tables& t, char* out, int64_t c0, int64_t c1,
                                             const uint32_t* base, const uint32_t* delta, uint32_t neg) {
  for (int64_t col = c0 + threadIdx.x; col < c1; col += blockDim.x) {
    const bool ok = col < t.vocab && ((mask_word(base, delta, col >> 5) >> (col & 31)) & 1u);
    if (!ok) {
      if (ELT == 2)
        *reinterpret_cast<uint16_t*>(out + 2 * col) = static_cast<uint16_t>(neg);
      else
        *reinterpret_cast<uint32_t*>(out + 4 * col) = neg;
    }
  }
}

// ---------------------------------------------------------------------------------------
// Logit policies of apply_mask: escape bias and release (csrc/engine.cu:2416-2552 of the
// reference).  A row's CTA runs them between building its mask and writing its -inf:
// warp 0 adds the bias, then the whole CTA reads the row once for its allowed mass and, if
// the row is released, replaces the mask it writes with the escape marker's next tokens.

// One logit as fp32 (ELT 2: bfloat16, or float16 when f16) and back, rounded to nearest.
template <int ELT>
__device__ __forceinline__ float load_logit(const char* at, bool f16) {
  if (ELT == 4) return *reinterpret_cast<const float*>(at);
  const uint16_t bits = *reinterpret_cast<const uint16_t*>(at);
  return f16 ? __half2float(__ushort_as_half(bits)) : __uint_as_float(static_cast<uint32_t>(bits) << 16);
}

template <int ELT>
__device__ __forceinline__ void store_logit(char* at, float value, bool f16) {
  if (ELT == 4)
    *reinterpret_cast<float*>(at) = value;
  else if (f16)
    *reinterpret_cast<__half*>(at) = __float2half_rn(value);
  else
    *reinterpret_cast<__nv_bfloat16*>(at) = __float2bfloat16_rn(value);
}

// A logit rounded to the row's element type (the value a 16-bit row holds).
template <int ELT>
__device__ __forceinline__ float rounded(float value, bool f16) {
  if (ELT == 4) return value;
  return f16 ? __half2float(__float2half_rn(value)) : __bfloat162float(__float2bfloat16_rn(value));
}

// One biased logit: its column and its value before and after.
struct BiasEdit {
  int32_t col;
  float before, after;
};
constexpr int32_t kMaxEdits = 64;  // edits a row records (more: its mass is read again whole)

// Warp: escape_bias added to the row's tokens that commit to the escape marker (all
// allowed, so none of the row's -inf writes touches them); with `edits`, lane 0 records
// each change there (count in *edit_count, which may exceed kMaxEdits).
template <int ELT>
__device__ void add_escape_bias(const Ctx& c, const XgState& s, char* out, int32_t cols, bool f16,
                                BiasEdit* edits = nullptr, int32_t* edit_count = nullptr) {
  for_each_escape_commit(c, s, [&](int32_t token) {
    if (c.w.leader() && token < cols) {
      char* at = out + static_cast<int64_t>(token) * ELT;
      const float before = load_logit<ELT>(at, f16);
      const float after = rounded<ELT>(before + c.t.escape_bias, f16);
      store_logit<ELT>(at, after, f16);
      if (edits) {
        const int32_t n = (*edit_count)++;
        if (n < kMaxEdits) edits[n] = BiasEdit{token, before, after};
      }
    }
  });
}

// A row's softmax mass in one pass: the top logit (lowest column among equal maxima), and
// the sums of exp(logit - anchor) over all columns and over the allowed ones.  The anchor
// is a value the pass has seen, at most kAnchorSpan below its top: it moves up (rescaling
// the sums) only when a value exceeds it by more, so a group's exponentials wait on
// nothing but that rare test, and no sum can overflow (128 K terms of at most e^64).  The
// release test reads the ratio allowed / all, which the anchor does not change.  exp(y)
// is 2^(y · log2 e) on the special-function unit (ex2.approx, relative error below 2^-22;
// results under 2^-126 flush to zero, below what any sum holding the anchor's own 1 can
// see).  The reference reads the row twice (the top first, then the sums with expf); the
// ratios agree to a few float roundings.
struct RowMass {
  float top;
  int32_t at;
  float anchor;
  float all, allowed;
};

constexpr float kLog2E = 1.4426950408889634f;  // log2(e)
constexpr float kAnchorSpan = 64.0f;

__device__ __forceinline__ float ex2(float y) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(y));
  return r;
}

__device__ __forceinline__ float exp_of(float y) { return ex2(y * kLog2E); }

// The anchor raised to `to` (a value above anchor + kAnchorSpan; the first finite value).
__device__ __forceinline__ void raise_anchor(RowMass& m, float to) {
  const float scale = m.anchor == -INFINITY ? 0.0f : exp_of(m.anchor - to);
  m.all *= scale;
  m.allowed *= scale;
  m.anchor = to;
}

// One column (the unaligned and ragged ends of a row).
__device__ __forceinline__ void mass_add(RowMass& m, float x, int32_t col, bool ok) {
  if (x > m.top) {  // NaN never rises
    m.top = x;
    m.at = col;
  }
  if (x > m.anchor + kAnchorSpan) raise_anchor(m, x);
  // below an anchor of -inf only -inf (adds 0) or NaN (carried, as the reference's sum carries it)
  const float e = m.anchor == -INFINITY ? (x != x ? x : 0.0f) : exp_of(x - m.anchor);
  m.all += e;
  if (ok) m.allowed += e;
}

__device__ __forceinline__ RowMass mass_merge(const RowMass& a, const RowMass& b) {
  const bool second = b.top > a.top || (b.top == a.top && b.at < a.at);
  const float anchor = fmaxf(a.anchor, b.anchor);
  const float fa = a.anchor == -INFINITY ? 0.0f : exp_of(a.anchor - anchor);
  const float fb = b.anchor == -INFINITY ? 0.0f : exp_of(b.anchor - anchor);
  return RowMass{second ? b.top : a.top, second ? b.at : a.at, anchor, a.all * fa + b.all * fb,
                 a.allowed * fa + b.allowed * fb};
}

// One 32-column group of a logits row (2·ELT 16-byte vectors; bits: its allowed columns)
// into the running mass: the group's maximum, the two rare tests (a new top, a raised
// anchor), then 32 independent exponentials summed as a tree.
template <int ELT, bool MASKED>
__device__ __forceinline__ void mass_group(RowMass& m, const uint4* v, int32_t col, uint32_t bits, bool f16) {
  float x[32];
#pragma unroll
  for (int32_t q = 0; q < 2 * ELT; ++q) {
    const uint32_t lanes[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
    for (int32_t j = 0; j < 16 / ELT; ++j) {
      float& y = x[q * (16 / ELT) + j];
      if (ELT == 4) {
        y = __uint_as_float(lanes[j]);
      } else {
        const uint32_t half = (lanes[j >> 1] >> (16 * (j & 1))) & 0xffffu;
        y = f16 ? __half2float(__ushort_as_half(static_cast<uint16_t>(half))) : __uint_as_float(half << 16);
      }
    }
  }
  float top = x[0];
#pragma unroll
  for (int32_t j = 1; j < 32; ++j) top = fmaxf(top, x[j]);  // NaN is passed over, as by ">"
  if (top > m.top) {
    int32_t first = 31;
#pragma unroll
    for (int32_t j = 31; j >= 0; --j)
      if (x[j] == top) first = j;
    m.top = top;
    m.at = col + first;
  }
  if (top > m.anchor + kAnchorSpan) raise_anchor(m, top);
  if (m.anchor == -INFINITY) {  // only -inf and NaN so far: NaN is carried
#pragma unroll
    for (int32_t j = 0; j < 32; ++j) {
      if (x[j] != x[j]) {
        m.all += x[j];
        if (MASKED && ((bits >> j) & 1u)) m.allowed += x[j];
      }
    }
    return;
  }
  const float shift = m.anchor * kLog2E;
#pragma unroll
  for (int32_t j = 0; j < 32; ++j) {
    const float e = ex2(fmaf(x[j], kLog2E, -shift));
    x[j] = e;  // reuse: the exponential of column j
  }
  float all[8], allowed[8];
#pragma unroll
  for (int32_t k = 0; k < 8; ++k) {
    all[k] = (x[k] + x[k + 8]) + (x[k + 16] + x[k + 24]);
    if (MASKED)
      allowed[k] = (((bits >> k) & 1u) ? x[k] : 0.0f) + (((bits >> (k + 8)) & 1u) ? x[k + 8] : 0.0f) +
                   ((((bits >> (k + 16)) & 1u) ? x[k + 16] : 0.0f) + (((bits >> (k + 24)) & 1u) ? x[k + 24] : 0.0f));
  }
  m.all += ((all[0] + all[1]) + (all[2] + all[3])) + ((all[4] + all[5]) + (all[6] + all[7]));
  if (MASKED)
    m.allowed += ((allowed[0] + allowed[1]) + (allowed[2] + allowed[3])) +
                 ((allowed[4] + allowed[5]) + (allowed[6] + allowed[7]));
}

constexpr int32_t kMassBatch = 4;  // 16-byte loads a thread issues before it uses them

// The mass passes stream a row through shared memory with cp.async: each thread owns the
// 32-column groups g = thread (mod threads) (one mask word each; 64 bytes of bf16, 128 of
// fp32) and keeps kRingBytes of them in flight in its own slots of the CTA's ring, so a
// CTA has ~64 KB of its row in flight instead of the few KB its registers could hold.
// Completion is the hardware's (cp.async.wait_group counts the thread's own copy groups);
// no thread waits on another.
constexpr int32_t kRingBytes = 256;  // per thread

__device__ __forceinline__ void async_copy16(void* to, const void* from) {
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(to));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(from) : "memory");
}
__device__ __forceinline__ void async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 32-column group g of the row (16-byte aligned) into `slot`.
template <int ELT>
__device__ __forceinline__ void copy_group(uint8_t* slot, const char* row, int32_t g) {
  const char* from = row + static_cast<int64_t>(g) * 32 * ELT;
#pragma unroll
  for (int32_t q = 0; q < 2 * ELT; ++q) async_copy16(slot + 16 * q, from + 16 * q);
}

// Per thread: the mass of the columns thread `thread` of `threads` takes: its 32-column
// groups of a 16-byte aligned row through its ring slots (`ring`: kRingBytes), then the
// ragged end; every column of an unaligned row one by one.  Allowed bits from base | delta
// when MASKED.
template <int ELT, bool MASKED>
__device__ RowMass thread_mass(const Tables& t, const char* out, int32_t cols, const uint32_t* base,
                               const uint32_t* delta, bool f16, int32_t thread, int32_t threads, uint8_t* ring) {
  constexpr bool masked = MASKED;
  RowMass m{-INFINITY, 0, -INFINITY, 0.0f, 0.0f};
  int32_t tail = 0;  // columns before it were read as whole groups
  if ((reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
    constexpr int32_t group_bytes = 32 * ELT, depth = kRingBytes / group_bytes;
    const int32_t groups = cols / 32;
#pragma unroll
    for (int32_t d = 0; d < depth; ++d) {  // always `depth` commits, so that the wait count holds
      const int32_t g = thread + d * threads;
      if (g < groups) copy_group<ELT>(ring + d * group_bytes, out, g);
      async_commit();
    }
    for (int32_t i = 0;; ++i) {
      const int32_t g = thread + i * threads;
      if (g >= groups) break;
      const uint32_t bits = masked ? mask_word(base, delta, g) : 0u;  // in flight during the wait
      uint8_t* slot = ring + (i % depth) * group_bytes;
      async_wait<depth - 1>();  // the oldest of the thread's groups has landed
      uint4 v[2 * ELT];
#pragma unroll
      for (int32_t q = 0; q < 2 * ELT; ++q) v[q] = *reinterpret_cast<const uint4*>(slot + 16 * q);
      mass_group<ELT, MASKED>(m, v, g * 32, bits, f16);
      const int32_t next = g + depth * threads;  // the slot's values are used: refill it
      if (next < groups) copy_group<ELT>(slot, out, next);
      async_commit();
    }
    async_wait<0>();
    tail = groups * 32;
  }
  for (int32_t col = tail + thread; col < cols; col += threads)
    mass_add(m, load_logit<ELT>(out + static_cast<int64_t>(col) * ELT, f16), col,
             masked && ((mask_word(base, delta, col >> 5) >> (col & 31)) & 1u));
  return m;
}

// The merge of a warp's masses, in every lane.
__device__ __forceinline__ RowMass warp_mass(RowMass m) {
#pragma unroll
  for (int32_t d = 16; d > 0; d >>= 1) {
    const RowMass o{__shfl_xor_sync(0xffffffffu, m.top, d), __shfl_xor_sync(0xffffffffu, m.at, d),
                    __shfl_xor_sync(0xffffffffu, m.anchor, d), __shfl_xor_sync(0xffffffffu, m.all, d),
                    __shfl_xor_sync(0xffffffffu, m.allowed, d)};
    m = mass_merge(m, o);
  }
  return m;
}

// Whether a row of this mass is released (csrc/engine.cu:2536-2552): its log allowed mass
// under the release mass, or (release_top) its top column disallowed; never for a row
// whose top is not finite (no defined distribution).
__device__ __forceinline__ bool released_by(const Tables& t, const RowMass& r, const uint32_t* base,
                                            const uint32_t* delta) {
  if (!isfinite(r.top)) return false;
  const bool top_allowed = (mask_word(base, delta, r.at >> 5) >> (r.at & 31)) & 1u;
  return (t.release_top && !top_allowed) || logf(r.allowed) - logf(r.all) < t.release_log_mass;
}

// Whole CTA (every thread gets the same answer): whether the row, columns [0, cols) of the
// served vocabulary under the mask base | delta, is released (csrc/engine.cu:2479-2552),
// from one pass over the row.
template <int ELT>
__device__ bool release_row(const Tables& t, const char* out, int32_t cols, const uint32_t* base,
                            const uint32_t* delta, bool f16, uint8_t* ring) {
  __shared__ RowMass partial[32];
  const RowMass m = warp_mass(thread_mass<ELT, true>(t, out, cols, base, delta, f16, threadIdx.x, blockDim.x,
                                                     ring + threadIdx.x * kRingBytes));
  const int32_t warps = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = m;
  __syncthreads();
  RowMass r = partial[0];
  for (int32_t w = 1; w < warps; ++w) r = mass_merge(r, partial[w]);
  __syncthreads();  // partial may be reused by the caller's next row
  return released_by(t, r, base, delta);
}

// Per thread: the sum of exp(logit - anchor) over the allowed columns among the 32-column
// groups thread `thread` of `threads` takes (their mask words loaded kMassBatch at a time;
// only groups holding an allowed column are read), then the ragged end.
template <int ELT>
__device__ float thread_allowed_sum(const Tables& t, const char* out, int32_t cols, const uint32_t* base,
                                    const uint32_t* delta, float anchor, bool f16, int32_t thread, int32_t threads) {
  constexpr int32_t per = 16 / ELT;
  const int32_t groups = (reinterpret_cast<uintptr_t>(out) & 15u) == 0 ? cols / 32 : 0;
  const float shift = anchor * kLog2E;
  float sum = 0.0f;
  for (int32_t g0 = thread; g0 < groups; g0 += threads * kMassBatch) {
    uint32_t bits[kMassBatch];
#pragma unroll
    for (int32_t b = 0; b < kMassBatch; ++b) {
      const int32_t g = g0 + b * threads;
      bits[b] = g < groups ? mask_word(base, delta, g) : 0u;
    }
#pragma unroll 1
    for (int32_t b = 0; b < kMassBatch; ++b) {
      if (bits[b] == 0u) continue;
      const int32_t g = g0 + b * threads;
      uint4 v[2 * ELT];
#pragma unroll
      for (int32_t q = 0; q < 2 * ELT; ++q)
        v[q] = *reinterpret_cast<const uint4*>(out + static_cast<int64_t>(g) * 32 * ELT + 16 * q);
#pragma unroll
      for (int32_t q = 0; q < 2 * ELT; ++q) {
        const uint32_t lanes[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
        for (int32_t j = 0; j < per; ++j) {
          if (!((bits[b] >> (q * per + j)) & 1u)) continue;
          float x;
          if (ELT == 4) {
            x = __uint_as_float(lanes[j]);
          } else {
            const uint32_t half = (lanes[j >> 1] >> (16 * (j & 1))) & 0xffffu;
            x = f16 ? __half2float(__ushort_as_half(static_cast<uint16_t>(half))) : __uint_as_float(half << 16);
          }
          sum += ex2(fmaf(x, kLog2E, -shift));
        }
      }
    }
  }
  for (int32_t col = groups * 32 + thread; col < cols; col += threads)
    if ((mask_word(base, delta, col >> 5) >> (col & 31)) & 1u)
      sum += exp_of(load_logit<ELT>(out + static_cast<int64_t>(col) * ELT, f16) - anchor);
  return sum;
}

// Whole CTA: whether the row is released, given `early`: the row's top and sum of all
// columns, read before its bias (by the warps idle during the state machine), and the
// bias edits since.  An edit at or above the top (or more edits than were recorded) leaves
// the top unknown: the row is read again whole.  Otherwise the sum takes each edit's
// change and the allowed sum is read from the vectors holding allowed columns only.
template <int ELT>
__device__ bool release_row_after(const Tables& t, const char* out, int32_t cols, const uint32_t* base,
                                  const uint32_t* delta, bool f16, RowMass early, const BiasEdit* edits,
                                  int32_t edit_count, uint8_t* ring) {
  __shared__ float partial[32];
  bool whole = edit_count > kMaxEdits || !isfinite(early.top);
  for (int32_t e = 0; e < edit_count && e < kMaxEdits && !whole; ++e) {
    const BiasEdit& x = edits[e];
    if (!(x.before < early.top && x.after < early.top)) whole = true;  // (NaN: whole too)
    else early.all += exp_of(x.after - early.anchor) - exp_of(x.before - early.anchor);
  }
  if (whole) return release_row<ELT>(t, out, cols, base, delta, f16, ring);  // block-uniform
  float sum = thread_allowed_sum<ELT>(t, out, cols, base, delta, early.anchor, f16, threadIdx.x, blockDim.x);
#pragma unroll
  for (int32_t d = 16; d > 0; d >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, d);
  const int32_t warps = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = sum;
  __syncthreads();
  float allowed = 0.0f;
  for (int32_t w = 0; w < warps; ++w) allowed += partial[w];
  __syncthreads();
  early.allowed = allowed;
  return released_by(t, early, base, delta);
}

// Whole CTA: `words` (words_padded, shared) becomes the mask of the escape marker's next
// tokens from byte position pos.
__device__ void released_mask(const Tables& t, int32_t pos, uint32_t* words) {
  for (int32_t k = threadIdx.x; k < t.words_padded; k += blockDim.x) words[k] = 0u;
  __syncthreads();
  const int32_t a = delim_begin(t.escape, pos), b = delim_end(t.escape, pos);
  for (int32_t i = a + threadIdx.x; i < b; i += blockDim.x) {
    const int32_t token = t.escape.tok[i];
    atomicOr(words + (token >> 5), 1u << (token & 31));
  }
  __syncthreads();
}

// apply_mask: -inf into every disallowed column of every row of an active, non-error
// slot; a CTA owns a 1/chunks share of one row.  ELT: element bytes (2 or 4); neg: the
// element's -inf bit pattern.
template <int ELT>
__global__ void __launch_bounds__(kApplyThreads, 4)
    apply_kernel(const __grid_constant__ Tables t, char* logits, int32_t cols, int64_t stride,
                 const int32_t* row_slots, int32_t chunks, int32_t max_slots, uint32_t neg) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // masks of a preceding step kernel are complete
  const int32_t row = blockIdx.x / chunks;
  const int32_t chunk = blockIdx.x - row * chunks;
  const int32_t slot = row_slots[row];
  if (slot < 0 || slot >= max_slots || !t.active[slot]) return;
  const uint32_t* base = t.base[slot];
  const uint32_t* delta = t.delta[slot];
  if (base == nullptr && delta == nullptr) return;  // error phase: untouched
  char* out = logits + static_cast<int64_t>(row) * stride * ELT;
  if ((reinterpret_cast<uintptr_t>(out) & 15u) != 0) {
    const int64_t per = (cols + chunks - 1) / chunks;
    const int64_t c0 = chunk * per;
    apply_scalar<ELT>(t, out, c0, c0 + per < cols ? c0 + per : cols, base, delta, neg);
    return;
  }
  if (const int32_t* list = delta == nullptr ? sparse_row(t, base) : nullptr) {  // few blocked tokens
    apply_sparse<ELT>(t, out, cols, list, neg, chunk == 0, chunk == 0 ? 0 : cols, cols);
    return;
  }
  const int32_t segments = (cols + 1023) >> 10;
  const int32_t share = (segments + chunks - 1) / chunks;
  const int32_t s0 = chunk * share;
  apply_segments<ELT>(t, out, cols, base, delta, neg, s0, s0 + share < segments ? s0 + share : segments,
                      threadIdx.x >> 5, blockDim.x >> 5, nullptr);
}

// ---------------------------------------------------------------------------------------
// Admission of one request into a slot (a warp; lane 0 writes the slot's buffers): begin or
// end, then anchors, then the KG version, then open_span, in the reference adapter's order
// (src/xgraph/vllm.py:569-605; begin = csrc/engine.cu:2027-2053, the rest 2840-2876, 2955).
// Returns false, touching nothing, when a field is out of range (counted in *faults, bit 1).
__device__ bool admit_slot(const Ctx& c, XgState& s, const XgAdmission& a, int32_t* faults) {
  const Tables& t = c.t;
  const int32_t lane = c.w.lane;
  const int32_t on = a.on, version = a.version, anchors = a.anchor_count;
  bool bad = version < 0 || version > t.versions || anchors < 0 || anchors > kMaxSet;
  if (!bad && on) {
    const int32_t k0 = lane, k1 = lane + 32;
    const int32_t r0 = k0 < anchors ? a.anchors[k0] : 0, p0 = k0 > 0 && k0 < anchors ? a.anchors[k0 - 1] : -1;
    const int32_t r1 = k1 < anchors ? a.anchors[k1] : 0, p1 = k1 < anchors ? a.anchors[k1 - 1] : -1;
    const bool wrong = (k0 < anchors && (r0 < 0 || r0 >= t.ent.count || r0 <= p0)) ||
                       (k1 < anchors && (r1 < 0 || r1 >= t.ent.count || r1 <= p1));
    bad = __any_sync(0xffffffffu, wrong);
  }
  if (bad) {
    if (c.w.leader()) atomicOr(faults, 2);
    return false;
  }
  int32_t* words = reinterpret_cast<int32_t*>(&s);
#pragma unroll
  for (int32_t k = 0; k < XG_STATE_INTS; ++k) words[k] = 0;
  if (on) {
    if (lane < anchors) c.mem[kMemReachedRows + lane] = a.anchors[lane];
    if (lane + 32 < anchors) c.mem[kMemReachedRows + lane + 32] = a.anchors[lane + 32];
  }
  if (c.w.leader()) {
    c.mem[kMemFacts] = c.mem[kMemFrontier] = 0;
    c.mem[kMemReached] = on ? anchors : 0;
    c.mem[kMemVersion] = on ? version : 0;
    c.mem[kMemPendingLo] = -1;
    t.cursors[c.slot] = -1;
    t.active[c.slot] = on ? 1 : 0;
    t.base[c.slot] = t.free_mask;
    t.delta[c.slot] = nullptr;
    if (t.stop_on) t.stop_on[c.slot] = 0;
  }
  __syncwarp();
  if (on && a.open_span) open_span(c, s);  // reads the anchors and version just written
  return true;
}

// admit: one warp per admission; the slot's state and mask are rebuilt.
__global__ void __launch_bounds__(32)
    admit_kernel(const __grid_constant__ Tables t, const XgAdmission* admit, int32_t max_slots, int32_t* faults) {
  __shared__ WarpShared shared;
  const XgAdmission& a = admit[blockIdx.x];
  const int32_t slot = a.slot;
  if (slot < 0 || slot >= max_slots) {
    if (threadIdx.x == 0) atomicOr(faults, 2);
    return;
  }
  Ctx c = make_ctx(t, slot, shared);
  XgState s;
  if (!admit_slot(c, s, a, faults)) return;
  store_state(t, slot, s);
  if (a.on) build_mask(c, s);
}

// ---------------------------------------------------------------------------------------
// The fused decoding step: sync + apply_mask for the step where logits row i belongs to
// slots[i] (no draft rows), with the step's admissions applied first.  Warp 0 of CTA i
// applies row i's admission (if any), consumes the slot's new history tokens and rebuilds
// its mask; then all warps of the CTA write the row's -inf.  One launch per decoding step;
// a row's stores overlap other rows' state-machine latency.  An admission whose slot is
// not a row of the step is applied by CTA (its index mod the grid) after its own row.

struct FusedArgs {
  StepArgs a;
  const XgAdmission* admit;  // this step's admissions (distinct slots) or null
  int32_t admit_count;
  int32_t max_slots;
  char* logits;
  int64_t stride;
  int32_t cols;
  uint32_t neg;
  int32_t* faults;
};

template <int ELT>
__global__ void __maxnreg__(kFusedRegisters)
    sync_apply_kernel(const __grid_constant__ Tables t, const __grid_constant__ FusedArgs f) {
  __shared__ WarpShared shared;
  __shared__ MaskRef use;                               // the mask this CTA applies
  __shared__ int32_t escape_at;                         // release: the row's escape position, or -1
  __shared__ RowMass early_mass[kFusedThreads / 32 - 1];  // release: warps 1..7's pass over the row
  __shared__ int32_t early_ready;                       //   done (the row was in a span before the step)
  __shared__ BiasEdit edits[kMaxEdits];                 // the escape bias's tokens and changes to the row
  __shared__ int32_t edit_count;
  __shared__ int32_t delim0[kDelimCopy];                // tokens that start each delimiter
  __shared__ __align__(128) uint32_t blocked_run[kBlockedRunWords];
  __shared__ int32_t prewritten;                        // the row's columns outside rel_any were written early
  extern __shared__ __align__(16) uint32_t composed[];  // [words_padded]: a delta built this step
  const int32_t i = blockIdx.x;
  const int32_t slot = f.a.slots[i];
  const bool valid = slot >= 0 && slot < f.max_slots;
  const bool f16 = ELT == 2 && f.neg == 0xfc00u;
  // Warp 0's loads of the slot's cursor, lengths and state are issued together with the
  // active flag (and the admission search) rather than after the branch on it.
  const int32_t was_on = valid ? t.active[slot] : 0;
  if (!was_on && f.admit_count == 0) return;  // block-uniform: inactive rows are neither advanced nor masked
  int32_t found = -1, cursor = 0, end = 0, prompt = 0;
  bool bias_row = false;  // warp 0: the row has more bias tokens than the list holds
  XgState s;
  if (threadIdx.x < 32 && valid) {
    // the first 32 admissions' slots load with the state (one round trip for both)
    const int32_t lane = threadIdx.x;
    const int32_t listed = lane < f.admit_count ? f.admit[lane].slot : -1;
    const int32_t stored = t.cursors[slot];
    prompt = f.a.prompt_len[slot];
    end = f.a.total_len[slot];
    s = load_state(t, slot);
    cursor = stored < 0 ? prompt : stored;
    uint32_t ballot = __ballot_sync(0xffffffffu, listed == slot);
    int32_t at = 0;
#pragma unroll 1
    while (ballot == 0u && at + 32 < f.admit_count) {
      at += 32;
      ballot = __ballot_sync(0xffffffffu, at + lane < f.admit_count && f.admit[at + lane].slot == slot);
    }
    if (ballot) found = at + __ffs(ballot) - 1;
  }
  uint32_t* const own = t.masks + static_cast<int64_t>(valid ? slot : 0) * t.words_padded;  // the slot's delta row
  // Warps 1..7, idle while warp 0 runs the state machine, clear the shared delta row, fill
  // the -inf run and copy the delimiters' start tokens, then arrive at barrier 1, which
  // warp 0 waits at before it composes the mask.
  const int32_t c0 = t.closer.at[1] - t.closer.at[0], c1 = t.separator.at[1] - t.separator.at[0];
  const int32_t c2 = t.escape.at[1] - t.escape.at[0];
  const bool copied = c0 + c1 + c2 <= kDelimCopy;
  if (threadIdx.x >= 32) {
    uint4* to = reinterpret_cast<uint4*>(composed);
    for (int32_t k = threadIdx.x - 32; k < (t.words_padded >> 2); k += blockDim.x - 32) to[k] = make_uint4(0u, 0u, 0u, 0u);
    fill_blocked_run<ELT>(blocked_run, f.neg, 32);
    if (copied) {
      for (int32_t k = threadIdx.x - 32; k < c0 + c1 + c2; k += blockDim.x - 32)
        delim0[k] = k < c0 ? t.closer.tok[t.closer.at[0] + k]
                           : k < c0 + c1 ? t.separator.tok[t.separator.at[0] + k - c0]
                                         : t.escape.tok[t.escape.at[0] + k - c0 - c1];
    }
    // Early writes.  Some rows' next mask is known, before the state machine runs, to lie
    // inside rel_any, every relation label token and delimiter token (~100 columns of a
    // 128 K vocabulary): every column outside it is -inf whatever the state machine finds,
    // and these warps write those columns now, while warp 0 runs the row's transitions (for
    // a relation label the longest: the next path frontier) and while the memory system is
    // still quiet; after the mask only rel_any's own columns remain.  With one new token and
    // no admission, that is (a) a relation-segment row whose token continues no delimiter
    // and is allowed by the slot's recorded mask: the token only narrows the relation label
    // (advance_span neither closes, separates, escapes nor errs), so the row stays in its
    // relation segment; (b) a subject (or path relation) row whose token completes the
    // separator and not the closer: next_segment moves it into a relation segment.  (A row
    // opening a span is not written early: its label-root mask leaves ~half the vocabulary
    // scattered, whose partial-line stores took ~23 us however early they started.)
    // Not with release, whose mass pass reads the row first.  The last warp decides, reading
    // the slot's state, cursor and recorded mask before it arrives at barrier 1: warp 0
    // writes none of them before that barrier (an admitted row, whose admission warp 0
    // applies earlier, is never written early).
    if (threadIdx.x >= blockDim.x - 32) {
      bool early_write = false;
      char* out_row = f.logits + static_cast<int64_t>(i) * f.stride * ELT;
      if (was_on && !t.release_on && t.dstep != nullptr && t.rel_any_count > 0 &&
          (reinterpret_cast<uintptr_t>(out_row) & 15u) == 0) {
        const int32_t lane = threadIdx.x & 31;
        const XgState* stored = t.states + slot;
        const int32_t phase = stored->phase, segment = stored->segment, answered = stored->answer_complete;
        const int32_t flags = stored->flags, close_pos = stored->close_pos, sep_pos = stored->sep_pos;
        const int32_t recorded = t.cursors[slot], first = f.a.prompt_len[slot], last = f.a.total_len[slot];
        const uint32_t* base0 = t.base[slot];
        const uint32_t* delta0 = t.delta[slot];
        bool admitted = false;
#pragma unroll 1
        for (int32_t at = 0; at < f.admit_count; at += 32)
          admitted |= __any_sync(0xffffffffu, at + lane < f.admit_count && f.admit[at + lane].slot == slot);
        const int32_t cursor0 = recorded < 0 ? first : recorded;
        if (!admitted && !answered && cursor0 + 1 == last) {
          const int32_t token = f.a.history[f.a.stride * slot + cursor0];
          if (token >= 0 && token < t.vocab && phase == kSpan) {
            const uint64_t packed = t.dstep[token];
            // delim_next over the packed word: the next byte position of delimiter branch
            // `offset + at`, or -1 (advance_span's reads, in its order)
            auto next = [&](int32_t offset, int32_t at) {
              const int32_t n = static_cast<int32_t>((packed >> (4 * (offset + at))) & 15u);
              return n ? n : -1;
            };
            const int32_t close = close_pos > 0 ? next(0, close_pos) : (flags & kMayClose) ? next(0, 0) : -1;
            const int32_t sep = sep_pos > 0 && !(flags & kStop) ? next(t.closer.len, sep_pos)
                                : (flags & kMaySep) ? next(t.closer.len, 0) : -1;
            if (segment == kRelation && packed == 0u &&
                ((mask_word(base0, delta0, token >> 5) >> (token & 31)) & 1u))
              early_write = true;
            else if (((segment == kSubject && stored->op == 0) || (segment == kRelation && t.paths)) &&
                     close != t.closer.len && sep == t.separator.len)
              early_write = true;
          }
        }
      }
      if (threadIdx.x == blockDim.x - 32) prewritten = early_write;
    }
    __syncwarp();
    asm volatile("bar.arrive 1, %0;" ::"r"(blockDim.x) : "memory");
    // Release reads the whole logits row of a span row.  For a row that was in a span
    // before this step's tokens (most span rows of a step; 16-byte aligned), these warps
    // start the row into L2 (bulk prefetches of 32 KB pieces, hints only) and take its top
    // and the sum over all its columns now, while warp 0 runs the state machine; after the
    // mask only the allowed columns remain to be read (release_row_after).  Other rows take
    // the whole pass after the mask (also taking rows that stay in free text measured
    // slower: their reads compete with every row's -inf writes for HBM).
    const char* row = f.logits + static_cast<int64_t>(i) * f.stride * ELT;
    const int32_t served = min(f.cols, t.vocab);
    const bool early = t.release_on && was_on && t.states[slot].phase == kSpan &&
                       (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
    if (early) {
      const int64_t bytes = (static_cast<int64_t>(served) * ELT) & ~15ll;
      for (int64_t at = static_cast<int64_t>(threadIdx.x - 32) * 32768; at < bytes;
           at += static_cast<int64_t>(blockDim.x - 32) * 32768) {
        const uint32_t piece = static_cast<uint32_t>(bytes - at < 32768 ? bytes - at : 32768);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(row + at), "r"(piece) : "memory");
      }
    }
    // A relation label of a path (base KG): the next frontier reads each frontier entity's
    // relation runs and its edges' folded first rows, two dependent round trips deep in
    // warp 0's transition.  Start those lines into L1 now, one thread per entity (the
    // slot's stored state and frontier are read here; the lines are only hints, and every
    // address is checked to lie in its table).
    if (was_on) {
      const XgState* stored = t.states + slot;
      const int32_t* mem = t.memory + static_cast<int64_t>(slot) * t.memory_ints;
      if (t.paths && stored->phase == kSpan && stored->segment == kRelation && mem[kMemVersion] == 0) {
        const int32_t count = mem[kMemFrontier] < kMaxSet ? mem[kMemFrontier] : kMaxSet;
        for (int32_t k = threadIdx.x - 32; k < count; k += blockDim.x - 32) {
          const int32_t e = mem[kMemFrontierEnt + k];
          if (e < 0 || e >= t.entities) continue;
          const int32_t r0 = t.run_off[e], r1 = t.run_off[e + 1], e0 = t.adj_off[e], e1 = t.adj_off[e + 1];
          for (int32_t x = 2 * r0; x <= 2 * r1 + 1 && x < 2 * r0 + 4 * 32; x += 32) prefetch_l1(t.runs + x);
          for (int32_t x = e0; x < e1 && x < e0 + 8 * 32; x += 32) prefetch_l1(t.edge_first + x);
        }
      }
    }
    // warps 1..7 only: the -inf run is filled and the early-write decision made
    asm volatile("bar.sync 2, %0;" ::"r"(blockDim.x - 32) : "memory");
    if (prewritten) {
      apply_segments<ELT>(t, f.logits + static_cast<int64_t>(i) * f.stride * ELT, f.cols, t.rel_any, nullptr, f.neg, 0,
                          (f.cols + 1023) >> 10, (threadIdx.x >> 5) - 1, (blockDim.x >> 5) - 1, blocked_run);
    }
    if (early) {
      uint8_t* ring = reinterpret_cast<uint8_t*>(composed + t.words_padded) + threadIdx.x * kRingBytes;
      const RowMass m = warp_mass(thread_mass<ELT, false>(t, row, served, nullptr, nullptr, f16, threadIdx.x - 32,
                                                          blockDim.x - 32, ring));
      if ((threadIdx.x & 31) == 0) early_mass[(threadIdx.x >> 5) - 1] = m;
    }
    if (threadIdx.x == 32) early_ready = early;
  } else {
    Ctx c = make_ctx(t, valid ? slot : 0, shared);
    if (copied) c.delim0 = delim0;
    bool changed = false;
    int32_t on = was_on;
    if (found >= 0 && admit_slot(c, s, f.admit[found], f.faults)) {
      changed = true;
      on = f.admit[found].on;
      cursor = prompt;
    }
    if (on && cursor < end) {
      const int32_t* tokens = f.a.history + f.a.stride * slot;
      for (; cursor < end; ++cursor) {
        const int32_t token = tokens[cursor];  // in flight while the state's reads are started
        if (s.phase == kSpan) prefetch_span(c, s);
        advance_state(c, s, token);
      }
      changed = true;
    }
    __syncwarp();
    asm volatile("bar.sync 1, %0;" ::"r"(blockDim.x) : "memory");
    // (the slot's state, cursor and mask pointers are written only after barrier 1: the
    // early-write decision reads them before it)
    if (changed) store_state(t, slot, s);
    if (prewritten && !(s.phase == kSpan && s.segment == kRelation) && threadIdx.x == 0)
      atomicOr(f.faults, 4);  // an early-written row left the relation segment (never expected)
    if (!on) {
      if (threadIdx.x == 0) use = MaskRef{nullptr, nullptr};  // inactive: untouched
    } else if (changed) {
      // the delta is composed in shared memory (setting bits there is much cheaper than in
      // global memory); the CTA copies it to the slot's row below
      const MaskRef m = compose_mask(c, s, composed, true);
      if (threadIdx.x == 0) {
        t.base[slot] = m.base;
        t.delta[slot] = m.delta ? own : nullptr;
        use = m;
      }
    } else {  // no new token: the slot's recorded mask
      if (threadIdx.x == 0) use = MaskRef{t.base[slot], t.delta[slot]};
    }
    if (threadIdx.x == 0 && on) t.cursors[slot] = cursor;
    // logit policies of a span row: its escape position for release, and the tokens the
    // bias goes to (their logits change after the barrier, once warps 1..7 have read the
    // row; more than kMaxEdits tokens: warp 0 finds them again then)
    const bool policies = on && s.phase == kSpan && (t.release_on || t.escape_bias != 0.0f);
    int32_t commits = 0;
    if (policies && t.escape_bias != 0.0f) {
      for_each_escape_commit(c, s, [&](int32_t token) {
        if (threadIdx.x == 0 && commits < kMaxEdits) edits[commits].col = token;
        ++commits;
      });
    }
    bias_row = commits > kMaxEdits;
    if (threadIdx.x == 0) {
      escape_at = policies ? escape_position(t, s) : -1;
      edit_count = commits;
    }
  }
  __syncthreads();
  const uint32_t* base = use.base;
  const uint32_t* delta = use.delta;
  {
    // The mask rows the -inf writes read from global memory (a table row, or the slot's
    // recorded delta row), prefetched into L1 line by line now: the row's later rounds of
    // mask loads then hit L1 instead of each waiting on L2 or HBM.
    const int32_t lines = (t.words + 31) >> 5;  // 128-byte lines of a mask row
    for (int32_t k = threadIdx.x; k < lines; k += blockDim.x) {
      if (base) asm volatile("prefetch.global.L1 [%0];" ::"l"(base + 32 * k));
      if (delta && delta != composed) asm volatile("prefetch.global.L1 [%0];" ::"l"(delta + 32 * k));
    }
  }
  if (delta == composed) {  // keep the slot's delta row current for later readers
    const uint4* from = reinterpret_cast<const uint4*>(composed);
    uint4* to = reinterpret_cast<uint4*>(own);
    for (int32_t k = threadIdx.x; k < (t.words_padded >> 2); k += blockDim.x) to[k] = from[k];
  }
  char* const row_out = f.logits + static_cast<int64_t>(i) * f.stride * ELT;
  if (bias_row) {  // warp 0, more tokens than were listed (the slot's state is in its registers)
    const Ctx c = make_ctx(t, slot, shared);
    add_escape_bias<ELT>(c, s, row_out, f.cols, f16);
  } else if (static_cast<int32_t>(threadIdx.x) < edit_count) {  // one listed token per thread
    BiasEdit& e = edits[threadIdx.x];
    if (e.col < f.cols) {
      char* at = row_out + static_cast<int64_t>(e.col) * ELT;
      e.before = load_logit<ELT>(at, f16);
      e.after = rounded<ELT>(e.before + t.escape_bias, f16);
      store_logit<ELT>(at, e.after, f16);
    } else {
      e.before = e.after = 0.0f;  // past the row: no change (and past the mass's columns)
    }
  }
  // release (block-uniform): the released mask replaces the composed one in shared memory
  // for this call only (the barriers below order every thread's copy above before it)
  if (escape_at >= 0 && t.release_on) {
    __syncthreads();  // the bias is written and its edits recorded
    const int32_t served = min(f.cols, t.vocab);
    bool released;
    if (early_ready) {
      RowMass early = early_mass[0];
      for (int32_t w = 1; w < kFusedThreads / 32 - 1; ++w) early = mass_merge(early, early_mass[w]);
      released = release_row_after<ELT>(t, row_out, served, base, delta, f16, early, edits, edit_count,
                                        reinterpret_cast<uint8_t*>(composed + t.words_padded));
    } else {
      released = release_row<ELT>(t, row_out, served, base, delta, f16,
                                  reinterpret_cast<uint8_t*>(composed + t.words_padded));
    }
    if (released) {
      released_mask(t, escape_at, composed);
      base = nullptr;
      delta = composed;
    }
  }
  if (base != nullptr || delta != nullptr) {  // else inactive or error phase: untouched
    char* out = f.logits + static_cast<int64_t>(i) * f.stride * ELT;
    if ((reinterpret_cast<uintptr_t>(out) & 15u) != 0) {
      apply_scalar<ELT>(t, out, 0, f.cols, base, delta, f.neg);
    } else if (prewritten) {  // the columns outside rel_any are -inf already: its own tokens remain
      for (int32_t k = threadIdx.x; k < t.rel_any_count; k += blockDim.x) {
        const int32_t token = t.rel_any_tok[k];
        if (token < f.cols && !((mask_word(base, delta, token >> 5) >> (token & 31)) & 1u)) {
          if (ELT == 2)
            *reinterpret_cast<uint16_t*>(out + 2 * static_cast<int64_t>(token)) = static_cast<uint16_t>(f.neg);
          else
            *reinterpret_cast<uint32_t*>(out + 4 * static_cast<int64_t>(token)) = f.neg;
        }
      }
    } else if (const int32_t* list = delta == nullptr ? sparse_row(t, base) : nullptr) {  // few blocked tokens
      apply_sparse<ELT>(t, out, f.cols, list, f.neg, true, 0, f.cols);
    } else {
      // The whole mask row is staged in shared memory first (one round of loads for the
      // row), so the store loop below reads no global memory: a load issued behind the
      // CTA's own outstanding stores waits for them, and a label-root row's ~67 k partial
      // stores held each of its later mask loads for microseconds.
      if (base != nullptr || delta != composed) {
        for (int32_t w = threadIdx.x; w < t.words_padded; w += blockDim.x)
          composed[w] = (base ? __ldg(base + w) : 0u) | (delta ? delta[w] : 0u);  // (delta may be composed)
        __syncthreads();
        base = nullptr;
        delta = composed;
      }
      apply_segments<ELT>(t, out, f.cols, base, delta, f.neg, 0, (f.cols + 1023) >> 10, threadIdx.x >> 5,
                          blockDim.x >> 5, blocked_run);
    }
  }
  // admissions whose slot is not a row of this step (CTA i takes i, i + grid, ...)
  if (threadIdx.x < 32) {
#pragma unroll 1
    for (int32_t j = i; j < f.admit_count; j += gridDim.x) {
      const int32_t other = f.admit[j].slot;
      const bool row = warp_any(Warp{static_cast<int32_t>(threadIdx.x)}, 0, f.a.count,
                                [&](int32_t r) { return f.a.slots[r] == other; });
      if (row) continue;
      if (other < 0 || other >= f.max_slots) {
        if (threadIdx.x == 0) atomicOr(f.faults, 2);
        continue;
      }
      Ctx c = make_ctx(t, other, shared);
      XgState x;
      if (!admit_slot(c, x, f.admit[j], f.faults)) continue;
      store_state(t, other, x);
      if (f.admit[j].on) build_mask(c, x);
    }
  }
}

// Speculative draft rows (apply_mask with local_pos and input_ids): a request owns
// consecutive logits rows, one per draft position; row r at offset k = local_pos[r] is
// masked as if the tokens fed at the request's rows r - k + 1 .. r (input_ids) had been
// committed to slot row_slots[r], in scratch: a copy of the slot's memory row and a mask
// row of its own (src/xgraph/engine.py:1012-1031, csrc/engine.cu:2353-2360).  The slot's
// state and memory do not move.  A row whose drafts reach the error phase, or whose offset
// reaches before the first row, is left untouched.  Offset 0 reads the slot's own mask.
struct DraftArgs {
  const int32_t* row_slots;
  const int32_t* local_pos;
  const int32_t* input_ids;
  int32_t max_slots;
  int32_t* scratch_memory;  // [rows, memory_ints]
  uint32_t* scratch_masks;  // [rows, words_padded]
};

// Scratch bytes per draft row: its memory row and its mask row (both 16-byte multiples).
inline int64_t draft_row_bytes(const Tables& t) {
  return (static_cast<int64_t>(t.memory_ints) + t.words_padded) * 4;
}

template <int ELT>
__global__ void __launch_bounds__(kFusedThreads)
    draft_apply_kernel(const __grid_constant__ Tables t, const DraftArgs d, char* logits, int32_t cols,
                       int64_t stride, uint32_t neg) {
  __shared__ WarpShared shared;
  __shared__ MaskRef mask;
  __shared__ int32_t escape_at;                         // release: the row's escape position, or -1
  extern __shared__ __align__(16) uint32_t released[];  // release on: [words_padded], then the mass ring
  const int32_t row = blockIdx.x;
  const int32_t slot = d.row_slots[row];
  if (slot < 0 || slot >= d.max_slots || !t.active[slot]) return;  // block-uniform
  const bool f16 = ELT == 2 && neg == 0xfc00u;
  const bool policies = t.release_on || t.escape_bias != 0.0f;
  char* out = logits + static_cast<int64_t>(row) * stride * ELT;
  if (threadIdx.x < 32) {
    const int32_t lane = threadIdx.x;
    const int32_t k = d.local_pos ? d.local_pos[row] : 0;
    MaskRef m{nullptr, nullptr};
    int32_t at = -1;
    // the logit policies of a span row: its escape position for release, and the bias now
    auto policy = [&](const Ctx& c, const XgState& s) {
      if (!policies || s.phase != kSpan) return;
      at = escape_position(t, s);
      if (t.escape_bias != 0.0f) add_escape_bias<ELT>(c, s, out, cols, f16);
    };
    if (k == 0) {
      m = MaskRef{t.base[slot], t.delta[slot]};
      if (policies) policy(make_ctx(t, slot, shared), t.states[slot]);
    } else if (k > 0 && k <= row) {
      int32_t* memory = d.scratch_memory + static_cast<int64_t>(row) * t.memory_ints;
      const int32_t* own = t.memory + static_cast<int64_t>(slot) * t.memory_ints;
#pragma unroll 1
      for (int32_t i = lane; i < t.memory_ints; i += 32) memory[i] = own[i];
      __syncwarp();
      Ctx c{t, Warp{lane}, slot, memory, shared.top, shared.scratch};
      XgState s = t.states[slot];
#pragma unroll 1
      for (int32_t j = 1; j <= k && s.phase != kError; ++j) advance_state(c, s, d.input_ids[row - k + j]);
      if (s.phase != kError) {
        m = compose_mask(c, s, d.scratch_masks + static_cast<int64_t>(row) * t.words_padded);
        policy(c, s);
      }
    }
    if (lane == 0) {
      mask = m;
      escape_at = at;
    }
  }
  __syncthreads();
  MaskRef m = mask;
  if (m.base == nullptr && m.delta == nullptr) return;  // error: untouched
  if (escape_at >= 0 && t.release_on &&
      release_row<ELT>(t, out, min(cols, t.vocab), m.base, m.delta, f16,
                       reinterpret_cast<uint8_t*>(released + t.words_padded))) {
    released_mask(t, escape_at, released);
    m = MaskRef{nullptr, released};
  }
  if ((reinterpret_cast<uintptr_t>(out) & 15u) != 0) {
    apply_scalar<ELT>(t, out, 0, cols, m.base, m.delta, neg);
    return;
  }
  apply_segments<ELT>(t, out, cols, m.base, m.delta, neg, 0, (cols + 1023) >> 10, threadIdx.x >> 5, blockDim.x >> 5,
                      nullptr);
}

// Engine set-up, one CTA: the write planning tables derived from the packed ones
// (Tables::rel_any, rel_any_tok, sparse, free_sparse, esc_sparse).  rel_any and out[0..2]
// arrive zeroed; out[0] = how many tokens rel_any holds, out[1] / out[2] = the free /
// escaped rows that have a sparse list.
__global__ void __launch_bounds__(1024) derive_kernel(const __grid_constant__ Tables t, uint32_t* rel_any,
                                                      int32_t* rel_any_tok, int32_t* sparse, int32_t* out,
                                                      int32_t free_rows, int32_t esc_rows) {
  __shared__ int32_t blocked;
  auto mark = [&](uint32_t* row, int32_t token) {
    if (token >= 0 && token < t.vocab) atomicOr(row + (token >> 5), 1u << (token & 31));
  };
  const int32_t relation_tokens = t.rel.off[t.rel.count];
  for (int32_t k = threadIdx.x; k < relation_tokens; k += blockDim.x) mark(rel_any, t.rel.tok[k]);
  for (const Delim* d : {&t.closer, &t.separator, &t.escape}) {
    const int32_t n = d->off[d->len];
    for (int32_t k = threadIdx.x; k < n; k += blockDim.x) mark(rel_any, d->tok[k]);
  }
  __syncthreads();
  for (int32_t w = threadIdx.x; w < t.words; w += blockDim.x) {
    for (uint32_t bits = rel_any[w]; bits; bits &= bits - 1u) rel_any_tok[atomicAdd(out, 1)] = 32 * w + __ffs(bits) - 1;
  }
  const uint32_t last = (t.vocab & 31) ? (1u << (t.vocab & 31)) - 1u : ~0u;  // the last word's vocabulary bits
  for (int32_t which = 0; which < 2; ++which) {
    const uint32_t* rows = which == 0 ? t.free_mask : t.esc_mask;
    const int32_t count = min(which == 0 ? free_rows : esc_rows, 32);
    for (int32_t p = 0; p < count; ++p) {
      const uint32_t* row = rows + static_cast<int64_t>(p) * t.words_padded;
      int32_t* list = sparse + (32 * which + p) * (1 + kSparseBlocked);
      if (threadIdx.x == 0) blocked = 0;
      __syncthreads();
      int32_t mine = 0;
      for (int32_t w = threadIdx.x; w < t.words; w += blockDim.x)
        mine += __popc(~row[w] & (w + 1 < t.words ? ~0u : last));
      atomicAdd(&blocked, mine);
      __syncthreads();
      const int32_t total = blocked;
      __syncthreads();
      if (total > kSparseBlocked) continue;  // (block-uniform)
      if (threadIdx.x == 0) blocked = 0;
      __syncthreads();
      for (int32_t w = threadIdx.x; w < t.words; w += blockDim.x) {
        for (uint32_t bits = ~row[w] & (w + 1 < t.words ? ~0u : last); bits; bits &= bits - 1u)
          list[1 + atomicAdd(&blocked, 1)] = 32 * w + __ffs(bits) - 1;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        list[0] = total;
        out[1 + which] |= 1 << p;
      }
    }
  }
}

}  // namespace xg

// Scratch of xg_apply_mask_noalloc: one array in this library's device image per device,
// shared by every call on that device (its size is the entry point's whole budget).
constexpr int64_t kNoAllocScratchBytes = 8ll << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// ===========================================================================================
// C ABI

using namespace xg;

// One KG version as the host keeps it (so that the device arena can be rebuilt): its
// sorted edited subjects, their adjacency offsets (count + 1, from 0) and edges.
struct HostVersion {
  std::vector<int32_t> subjects, adjacency, relations, objects;
  bool live = false;
};

// The engine's KG versions on the device, outside the index blob so that versions can be
// added and dropped between steps: version id v owns subjects [range[2v-2], range[2v-1])
// of `subjects`, whose edges `adjacency` (absolute offsets, one past the last subject too)
// points into `relations` / `objects`.  Versions are appended; a dropped version's space is
// reclaimed when the arena is next rebuilt (on growth), from the host copies.
struct VersionArena {
  int32_t* range = nullptr;
  int32_t* subjects = nullptr;
  int32_t* adjacency = nullptr;
  int32_t* relations = nullptr;
  int32_t* objects = nullptr;
  int64_t id_cap = 0, subject_cap = 0, edge_cap = 0;
  int64_t subjects_used = 0, edges_used = 0;
  std::vector<HostVersion> versions;  // id - 1
};

struct XgEngine {
  int device = 0;
  int sm_count = 148;
  XgLayout layout{};
  XgOptions options{};
  int32_t max_sequences = 0;
  char* blob = nullptr;
  XgState* states = nullptr;
  int32_t* memory = nullptr;
  uint32_t* masks = nullptr;
  const uint32_t** base = nullptr;
  uint32_t** delta = nullptr;
  int32_t* cursors = nullptr;
  int32_t* active = nullptr;
  int32_t* tokens = nullptr;
  char* draft_scratch = nullptr;  // apply_mask's draft rows: [rows] memory rows, then [rows] mask rows
  int32_t draft_capacity = 0;     // rows it holds
  int32_t* faults = nullptr;      // device-side faults (xg_faults)
  XgAdmission* admissions = nullptr;  // staging of host admissions: max_sequences entries
  size_t composed_bytes = 0;      // sync_apply's dynamic shared memory: one mask row
  uint32_t* rel_any = nullptr;    // derived tables (derive_kernel): relation-segment superset mask,
  int32_t* rel_any_tok = nullptr; //   its tokens,
  int32_t* sparse = nullptr;      //   and the automaton rows' blocked-token lists
  uint32_t* successors = nullptr; // successor support's tables (xg_set_relation_successors)
  int32_t successor_tables = 0;
  // expressions (xg_set_expressions): one device buffer of the packed delimiter lists, then
  // the date table (entities, keys, first days, last days); the Tables fields they give
  int32_t* expr = nullptr;
  int64_t expr_delim_ints = 0;
  int32_t operator_count = 0;
  int32_t operator_lcp[kMaxOperators * kMaxOperators] = {};
  Delim operators[kMaxOperators] = {};
  Delim operand_sep{};
  int32_t date_count = 0;
  int32_t verdict_yes = -1, verdict_no = -1;
  // residual-goal STOP (xg_enable_stop): label words, and per slot: installed flag, relation
  // table, question word offsets and bytes
  int64_t* stop_label_off = nullptr;
  uint8_t* stop_label_words = nullptr;
  int32_t* stop_on = nullptr;
  int32_t* stop_rel = nullptr;
  int32_t* stop_woff = nullptr;
  uint8_t* stop_words = nullptr;
  VersionArena arena;
  Tables t{};
};

namespace {

thread_local std::string g_error;

int fail(int code, const std::string& message) {
  g_error = message;
  return code;
}

}  // namespace

// The adjacency builder (build.cu) reports its errors through the same last-error slot;
// not exported from the library.
extern "C" int xg_set_error(int code, const char* message) { return fail(code, message); }

namespace {

int cuda_fail(cudaError_t e, const char* what) {
  cudaGetLastError();  // clear a non-sticky error so the next call starts clean
  return fail(XG_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define XG_CUDA(call, what)                      \
  do {                                           \
    const cudaError_t e_ = (call);               \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

cudaStream_t as_stream(void* stream) { return reinterpret_cast<cudaStream_t>(stream); }

template <class T>
const T* at(const char* blob, int64_t offset) {
  return offset < 0 ? nullptr : reinterpret_cast<const T*>(blob + offset);
}

int check_layout(const XgLayout& l) {
  if (l.vocab <= 0 || l.words != (l.vocab + 31) / 32 || l.words_padded < l.words || l.words_padded % 4)
    return fail(XG_EINVAL, "layout: vocabulary and mask words disagree");
  if (l.entity_rows < 0 || l.relation_rows < 0 || l.entities < 0 || l.relations < 0 || l.versions < 0 ||
      l.wide_count < 0 || l.relation_words != (l.relations + 31) / 32)
    return fail(XG_EINVAL, "layout: negative or inconsistent table sizes");
  if (l.opener_len <= 0 || l.closer_len <= 0 || l.separator_len <= 0 || l.escape_len <= 0 ||
      l.opener_len > 127 || l.closer_len > 127)
    return fail(XG_EINVAL, "layout: delimiter lengths out of range");
  if (l.ent_cols < 1 || l.rel_cols < 1) return fail(XG_EINVAL, "layout: column tables missing");
  const int64_t required[] = {l.ent_tok, l.ent_off, l.ent_owner, l.rel_tok, l.rel_off, l.rel_owner,
                              l.ent_col, l.rel_col, l.ent_first, l.rel_first, l.row_degree, l.row_first,
                              l.run_off, l.runs, l.run_rel, l.edge_first,
                              l.ent_first_row, l.ent_rows_off, l.ent_rows, l.adj_off, l.edge_rel,
                              l.edge_obj, l.root_mask, l.free_next, l.free_mask, l.esc_next,
                              l.esc_mask, l.eos_mask, l.closer_off, l.closer_tok, l.closer_next,
                              l.separator_off, l.separator_tok, l.separator_next, l.escape_off,
                              l.escape_tok, l.escape_next, l.ver_off, l.ver_subj, l.ver_adj,
                              l.ver_edge_rel, l.ver_edge_obj};
  for (int64_t off : required)
    if (off < 0 || off > l.blob_bytes || off % 16) return fail(XG_EINVAL, "layout: table offset outside the blob");
  const int64_t optional[] = {l.sitelinks, l.row_sitelinks, l.kept_prefix, l.wide_keys, l.wide_masks, l.dstep};
  for (int64_t off : optional)
    if (off != -1 && (off < 0 || off > l.blob_bytes || off % 16))
      return fail(XG_EINVAL, "layout: optional table offset outside the blob");
  if (l.wide_count > 0 && (l.wide_keys < 0 || l.wide_masks < 0)) return fail(XG_EINVAL, "layout: wide masks missing");
  return XG_OK;
}

// The first CSR offsets of a delimiter's lists, read from the blob wherever it lives.
int fill_delimiter_offsets(Delim& d, const char* blob, int64_t offset, const void* host_blob) {
  const int32_t n = (d.len + 1) < 17 ? d.len + 1 : 17;
  for (int32_t k = 0; k < 17; ++k) d.at[k] = 0;
  if (host_blob) {
    std::memcpy(d.at, static_cast<const char*>(host_blob) + offset, n * sizeof(int32_t));
    return XG_OK;
  }
  XG_CUDA(cudaMemcpy(d.at, blob + offset, n * sizeof(int32_t), cudaMemcpyDeviceToHost), "delimiter offsets");
  return XG_OK;
}

void bind_versions(XgEngine* e) {
  const VersionArena& a = e->arena;
  e->t.ver_range = a.range;
  e->t.ver_subj = a.subjects;
  e->t.ver_adj = a.adjacency;
  e->t.ver_edge_rel = a.relations;
  e->t.ver_edge_obj = a.objects;
  e->t.versions = static_cast<int32_t>(a.versions.size());
}

// Append live version `id` at the arena's end (capacity checked by the caller).
int place_version(XgEngine* e, int32_t id, cudaStream_t stream) {
  VersionArena& a = e->arena;
  const HostVersion& v = a.versions[id - 1];
  const int64_t n = static_cast<int64_t>(v.subjects.size()), m = static_cast<int64_t>(v.relations.size());
  std::vector<int32_t> absolute(v.adjacency.size());
  for (size_t i = 0; i < absolute.size(); ++i) absolute[i] = static_cast<int32_t>(a.edges_used + v.adjacency[i]);
  const int32_t range[2] = {static_cast<int32_t>(a.subjects_used), static_cast<int32_t>(a.subjects_used + n)};
  // pageable sources: each copy is staged before the call returns, so the temporaries may go
  if (n) XG_CUDA(cudaMemcpyAsync(a.subjects + a.subjects_used, v.subjects.data(), n * 4, cudaMemcpyHostToDevice, stream),
                 "version upload");
  XG_CUDA(cudaMemcpyAsync(a.adjacency + a.subjects_used, absolute.data(), (n + 1) * 4, cudaMemcpyHostToDevice, stream),
          "version upload");
  if (m) {
    XG_CUDA(cudaMemcpyAsync(a.relations + a.edges_used, v.relations.data(), m * 4, cudaMemcpyHostToDevice, stream),
            "version upload");
    XG_CUDA(cudaMemcpyAsync(a.objects + a.edges_used, v.objects.data(), m * 4, cudaMemcpyHostToDevice, stream),
            "version upload");
  }
  XG_CUDA(cudaMemcpyAsync(a.range + 2 * (id - 1), range, sizeof(range), cudaMemcpyHostToDevice, stream), "version upload");
  a.subjects_used += n;
  a.edges_used += m;
  return XG_OK;
}

// A fresh arena holding every live version contiguously, with room for at least `ids`
// versions, `subjects` subjects and `edges` edges; the old buffers are freed in stream
// order (after the work already queued on `stream` that may read them).
int rebuild_versions(XgEngine* e, int64_t ids, int64_t subjects, int64_t edges, cudaStream_t stream) {
  VersionArena& a = e->arena;
  VersionArena fresh;
  fresh.versions.swap(a.versions);
  int64_t live_subjects = 0, live_edges = 0;
  for (const HostVersion& v : fresh.versions) {
    if (!v.live) continue;
    live_subjects += static_cast<int64_t>(v.subjects.size());
    live_edges += static_cast<int64_t>(v.relations.size());
  }
  fresh.id_cap = std::max<int64_t>({16, ids, 2 * a.id_cap});
  fresh.subject_cap = std::max<int64_t>({1024, subjects, live_subjects, 2 * a.subject_cap});
  fresh.edge_cap = std::max<int64_t>({4096, edges, live_edges, 2 * a.edge_cap});
  if (fresh.subject_cap + 1 > 0x7fffffff || fresh.edge_cap > 0x7fffffff)
    return fail(XG_EINVAL, "KG versions: more than 2^31 edited subjects or edges");
  cudaError_t err = cudaSuccess;
  auto alloc = [&](int32_t** p, int64_t count) {
    if (err == cudaSuccess) err = cudaMallocAsync(reinterpret_cast<void**>(p), count * sizeof(int32_t), stream);
  };
  alloc(&fresh.range, 2 * fresh.id_cap);
  alloc(&fresh.subjects, fresh.subject_cap);
  alloc(&fresh.adjacency, fresh.subject_cap + 1);
  alloc(&fresh.relations, fresh.edge_cap);
  alloc(&fresh.objects, fresh.edge_cap);
  if (err == cudaSuccess) err = cudaMemsetAsync(fresh.range, 0, 2 * fresh.id_cap * sizeof(int32_t), stream);
  if (err == cudaSuccess) err = cudaMemsetAsync(fresh.adjacency, 0, sizeof(int32_t), stream);
  if (err != cudaSuccess) {
    for (int32_t* p : {fresh.range, fresh.subjects, fresh.adjacency, fresh.relations, fresh.objects})
      if (p) cudaFreeAsync(p, stream);
    a.versions.swap(fresh.versions);
    cudaGetLastError();
    return fail(XG_ENOMEM, std::string("KG version arena: ") + cudaGetErrorString(err));
  }
  std::swap(a, fresh);  // `fresh` now holds the old buffers
  for (int32_t id = 1; id <= static_cast<int32_t>(a.versions.size()); ++id)
    if (a.versions[id - 1].live)
      if (int rc = place_version(e, id, stream)) return rc;
  for (int32_t* p : {fresh.range, fresh.subjects, fresh.adjacency, fresh.relations, fresh.objects})
    if (p) cudaFreeAsync(p, stream);
  bind_versions(e);
  return XG_OK;
}

// Host checks of one version's arrays (the layout build_kg_versions writes).
int check_version(const XgEngine* e, const int32_t* subjects, int32_t count, const int64_t* adjacency,
                  const int32_t* relations, const int32_t* objects) {
  if (count < 0 || (count > 0 && (!subjects || !adjacency))) return fail(XG_EINVAL, "KG version: null arrays");
  if (count > 0 && adjacency[0] != 0) return fail(XG_EINVAL, "KG version: adjacency must start at 0");
  if (count > 0 && adjacency[count] > 0 && (!relations || !objects)) return fail(XG_EINVAL, "KG version: null edges");
  for (int32_t i = 0; i < count; ++i) {
    if (subjects[i] < 0 || subjects[i] >= e->layout.entities || (i > 0 && subjects[i] <= subjects[i - 1]))
      return fail(XG_EINVAL, "KG version: subjects must be sorted, distinct entity positions");
    if (adjacency[i + 1] < adjacency[i]) return fail(XG_EINVAL, "KG version: adjacency must not decrease");
    for (int64_t k = adjacency[i]; k < adjacency[i + 1]; ++k) {
      if (relations[k] < 0 || relations[k] >= e->layout.relations || objects[k] < 0 ||
          objects[k] >= e->layout.entity_rows)
        return fail(XG_EINVAL, "KG version: an edge names no relation or label row of the index");
      if (k > adjacency[i] && (relations[k] < relations[k - 1] ||
                               (relations[k] == relations[k - 1] && objects[k] <= objects[k - 1])))
        return fail(XG_EINVAL, "KG version: a subject's edges must be sorted by (relation, object row), distinct");
    }
  }
  if (count > 0 && adjacency[count] > 0x7fffffff) return fail(XG_EINVAL, "KG version: too many edges");
  return XG_OK;
}

// Register a version (host arrays): the lowest dropped id is reused, else a new one.
int add_version(XgEngine* e, const int32_t* subjects, int32_t count, const int64_t* adjacency,
                const int32_t* relations, const int32_t* objects, cudaStream_t stream, int32_t* out) {
  if (int rc = check_version(e, subjects, count, adjacency, relations, objects)) return rc;
  VersionArena& a = e->arena;
  int32_t id = 1;
  while (id <= static_cast<int32_t>(a.versions.size()) && a.versions[id - 1].live) ++id;
  if (id > static_cast<int32_t>(a.versions.size())) a.versions.emplace_back();
  HostVersion& v = a.versions[id - 1];
  const int64_t edges = count > 0 ? adjacency[count] : 0;
  v.subjects.assign(subjects, subjects + count);
  v.adjacency.resize(static_cast<size_t>(count) + 1);
  for (int32_t i = 0; i <= count; ++i) v.adjacency[i] = count > 0 ? static_cast<int32_t>(adjacency[i]) : 0;
  v.relations.assign(relations, relations + edges);
  v.objects.assign(objects, objects + edges);
  v.live = true;
  int rc = XG_OK;
  if (id > a.id_cap || a.subjects_used + count + 1 > a.subject_cap || a.edges_used + edges > a.edge_cap)
    rc = rebuild_versions(e, id, a.subjects_used + count + 1, a.edges_used + edges, stream);
  else
    rc = place_version(e, id, stream);
  if (rc) {
    v = HostVersion{};
    return rc;
  }
  bind_versions(e);
  *out = id;
  return XG_OK;
}

// The expression tables' fields of Tables (all zero until xg_set_expressions).  Only these:
// the rest of Tables keeps what create bound (the delimiters' offsets among it).
void bind_expressions(XgEngine* e) {
  Tables& t = e->t;
  t.operator_count = e->operator_count;
  for (int32_t k = 0; k < kMaxOperators * kMaxOperators; ++k) t.operator_lcp[k] = e->operator_lcp[k];
  for (int32_t k = 0; k < kMaxOperators; ++k) t.operators[k] = e->operators[k];
  t.operand_sep = e->operand_sep;
  const int32_t* dates = e->expr ? e->expr + e->expr_delim_ints : nullptr;
  t.date_entities = dates;
  t.date_keys = dates ? dates + e->date_count : nullptr;
  t.date_lo = dates ? dates + 2 * e->date_count : nullptr;
  t.date_hi = dates ? dates + 3 * e->date_count : nullptr;
  t.date_count = e->date_count;
  t.verdict_yes = e->verdict_yes;
  t.verdict_no = e->verdict_no;
}

void bind_tables(XgEngine* e) {
  const XgLayout& l = e->layout;
  const char* b = e->blob;
  Tables& t = e->t;
  t.ent = Rows{at<int32_t>(b, l.ent_tok), at<int32_t>(b, l.ent_off), at<int32_t>(b, l.ent_owner), l.entity_rows,
               at<int32_t>(b, l.ent_col), at<int32_t>(b, l.ent_first), l.ent_cols};
  t.rel = Rows{at<int32_t>(b, l.rel_tok), at<int32_t>(b, l.rel_off), at<int32_t>(b, l.rel_owner), l.relation_rows,
               at<int32_t>(b, l.rel_col), at<int32_t>(b, l.rel_first), l.rel_cols};
  t.ent_first_row = at<int32_t>(b, l.ent_first_row);
  t.row_degree = at<int32_t>(b, l.row_degree);
  t.row_first = at<int32_t>(b, l.row_first);
  t.ent_rows_off = at<int32_t>(b, l.ent_rows_off);
  t.ent_rows = at<int32_t>(b, l.ent_rows);
  t.adj_off = at<int32_t>(b, l.adj_off);
  t.edge_rel = at<int32_t>(b, l.edge_rel);
  t.edge_obj = at<int32_t>(b, l.edge_obj);
  t.run_off = at<int32_t>(b, l.run_off);
  t.runs = at<int32_t>(b, l.runs);
  t.run_rel = at<int32_t>(b, l.run_rel);
  t.edge_first = at<int32_t>(b, l.edge_first);
  t.sitelinks = e->options.sitelinks_rank ? at<int32_t>(b, l.sitelinks) : nullptr;
  t.row_sitelinks = e->options.sitelinks_rank ? at<int32_t>(b, l.row_sitelinks) : nullptr;
  t.kept_prefix = at<int32_t>(b, l.kept_prefix);
  t.root_mask = at<uint32_t>(b, l.root_mask);
  t.wide_keys = at<int64_t>(b, l.wide_keys);
  t.wide_masks = at<uint32_t>(b, l.wide_masks);
  t.wide_count = l.wide_count;
  t.free_next = at<int8_t>(b, l.free_next);
  t.free_mask = at<uint32_t>(b, l.free_mask);
  t.esc_next = at<int8_t>(b, l.esc_next);
  t.esc_mask = at<uint32_t>(b, l.esc_mask);
  t.eos_mask = at<uint32_t>(b, l.eos_mask);
  t.closer = Delim{at<int32_t>(b, l.closer_off), at<int32_t>(b, l.closer_tok), at<int32_t>(b, l.closer_next), l.closer_len};
  t.separator = Delim{at<int32_t>(b, l.separator_off), at<int32_t>(b, l.separator_tok),
                      at<int32_t>(b, l.separator_next), l.separator_len};
  t.escape = Delim{at<int32_t>(b, l.escape_off), at<int32_t>(b, l.escape_tok), at<int32_t>(b, l.escape_next), l.escape_len};
  t.dstep = at<uint64_t>(b, l.dstep);
  bind_versions(e);
  t.vocab = l.vocab;
  t.words = l.words;
  t.words_padded = l.words_padded;
  t.entities = l.entities;
  t.relations = l.relations;
  t.relation_words = l.relation_words;
  const XgOptions& o = e->options;
  t.escapes = o.escapes;
  t.repeats = o.repeats;
  t.derivation = o.derivation || o.paths;
  t.paths = o.paths;
  t.bound_escapes = o.bound_escapes;
  t.committed = o.committed_paths;
  t.end_after_answer = o.end_after_answer;
  t.release_log_mass = o.release_log_mass;
  t.release_top = o.release_top != 0;
  t.release_on = o.release_top != 0 || o.release_log_mass > -INFINITY;
  t.escape_bias = o.escape_bias;
  t.relation_mode = o.relations;
  t.successors = e->successors;
  t.successor_tables = e->successor_tables;
  t.states = e->states;
  t.memory = e->memory;
  t.memory_ints = memory_ints_for(l.relation_words, o.expressions != 0);
  t.mem_operand = o.expressions ? memory_ints_for(l.relation_words, false) : 0;
  bind_expressions(e);
  t.masks = e->masks;
  t.base = e->base;
  t.delta = e->delta;
  t.cursors = e->cursors;
  t.active = e->active;
}

void release(XgEngine* e) {
  cudaFree(e->blob);
  cudaFree(e->states);
  cudaFree(e->memory);
  cudaFree(e->masks);
  cudaFree(const_cast<uint32_t**>(e->base));
  cudaFree(e->delta);
  cudaFree(e->cursors);
  cudaFree(e->active);
  cudaFree(e->tokens);
  cudaFree(e->draft_scratch);
  cudaFree(e->faults);
  cudaFree(e->stop_label_off);
  cudaFree(e->stop_label_words);
  cudaFree(e->stop_on);
  cudaFree(e->stop_rel);
  cudaFree(e->stop_woff);
  cudaFree(e->stop_words);
  cudaFree(e->admissions);
  cudaFree(e->rel_any);
  cudaFree(e->rel_any_tok);
  cudaFree(e->sparse);
  cudaFree(e->successors);
  cudaFree(e->expr);
  for (void* p : {static_cast<void*>(e->arena.range), static_cast<void*>(e->arena.subjects),
                  static_cast<void*>(e->arena.adjacency), static_cast<void*>(e->arena.relations),
                  static_cast<void*>(e->arena.objects)})
    cudaFree(p);
  delete e;
}

// The versions packed in the index blob become the arena's first ids (1..versions).
int load_blob_versions(XgEngine* e, const void* host_blob) {
  const XgLayout& l = e->layout;
  auto read = [&](int64_t offset, int64_t count, std::vector<int32_t>& out) -> int {
    out.resize(static_cast<size_t>(count));
    if (count == 0) return XG_OK;
    if (host_blob) {
      std::memcpy(out.data(), static_cast<const char*>(host_blob) + offset, count * sizeof(int32_t));
      return XG_OK;
    }
    XG_CUDA(cudaMemcpy(out.data(), e->blob + offset, count * sizeof(int32_t), cudaMemcpyDeviceToHost), "version read");
    return XG_OK;
  };
  std::vector<int32_t> off, subj, adj, rel, obj;
  if (int rc = read(l.ver_off, static_cast<int64_t>(l.versions) + 1, off)) return rc;
  const int64_t subjects = off.empty() ? 0 : off.back();
  if (int rc = read(l.ver_subj, subjects, subj)) return rc;
  if (int rc = read(l.ver_adj, subjects + 1, adj)) return rc;
  const int64_t edges = adj.empty() ? 0 : adj.back();
  if (int rc = read(l.ver_edge_rel, edges, rel)) return rc;
  if (int rc = read(l.ver_edge_obj, edges, obj)) return rc;
  VersionArena& a = e->arena;
  a.versions.assign(static_cast<size_t>(l.versions), HostVersion{});
  for (int32_t v = 0; v < l.versions; ++v) {
    HostVersion& h = a.versions[v];
    const int32_t s0 = off[v], s1 = off[v + 1];
    if (s0 < 0 || s1 < s0 || s1 > subjects) return fail(XG_EINVAL, "layout: version offsets out of order");
    h.subjects.assign(subj.begin() + s0, subj.begin() + s1);
    h.adjacency.resize(static_cast<size_t>(s1 - s0) + 1);
    for (int32_t i = s0; i <= s1; ++i) h.adjacency[i - s0] = adj[i] - adj[s0];
    h.relations.assign(rel.begin() + adj[s0], rel.begin() + adj[s1]);
    h.objects.assign(obj.begin() + adj[s0], obj.begin() + adj[s1]);
    h.live = true;
  }
  return rebuild_versions(e, l.versions, subjects + 1, edges, nullptr);
}

int derive_tables(XgEngine* e);

int create(const void* blob, bool on_device, const XgLayout* layout, const XgOptions* options,
           int32_t max_sequences, XgEngine** out) {
  if (!blob || !layout || !options || !out) return fail(XG_EINVAL, "null argument");
  *out = nullptr;
  if (max_sequences < 1) return fail(XG_EINVAL, "max_sequences must be at least 1, got " + std::to_string(max_sequences));
  if (int rc = check_layout(*layout)) return rc;
  if (options->sitelinks_rank && (layout->sitelinks < 0 || layout->row_sitelinks < 0))
    return fail(XG_EINVAL, "the sitelink rank needs a KG index with sitelink counts");
  if (!(options->release_log_mass < 0.0f))
    return fail(XG_EINVAL, "release_log_mass must be the log of a mass in (0, 1), or -INFINITY when off");
  if ((options->release_top || options->release_log_mass > -INFINITY) && !options->escapes)
    return fail(XG_EINVAL, "release needs escapes: it releases to the escape marker");
  if (options->relations < 0 || options->relations > 2)
    return fail(XG_EINVAL, "relations must be 0 (frontier), 1 (vocabulary) or 2 (successor)");
  if (options->relations != 0 && !options->paths)
    return fail(XG_EINVAL, "weaker relations need path mode");
  if (options->relations == 2 && layout->relation_words > kScratchInts)
    return fail(XG_EINVAL, "successor support handles at most 10,304 relations");
  if (options->expressions && (!options->paths || !options->committed_paths))
    return fail(XG_EINVAL, "expressions need committed paths (committed_paths=True)");
  if (options->expressions && !options->escapes)
    return fail(XG_EINVAL, "expressions need escapes, the way out of an operand or relation");
  if (options->expressions && options->relations != 0)
    return fail(XG_EINVAL, "weaker relations need path mode without expressions or STOP");
  XgEngine* e = new XgEngine();
  e->layout = *layout;
  e->options = *options;
  e->max_sequences = max_sequences;
  cudaGetDevice(&e->device);
  cudaDeviceGetAttribute(&e->sm_count, cudaDevAttrMultiProcessorCount, e->device);
  const int64_t slots = max_sequences;
  const int32_t memory_ints = memory_ints_for(layout->relation_words, options->expressions != 0);
  cudaError_t err = cudaSuccess;
  auto alloc = [&](void** p, size_t bytes) {
    if (err == cudaSuccess) err = cudaMalloc(p, bytes > 0 ? bytes : 16);
  };
  alloc(reinterpret_cast<void**>(&e->blob), static_cast<size_t>(layout->blob_bytes));
  alloc(reinterpret_cast<void**>(&e->states), slots * sizeof(XgState));
  alloc(reinterpret_cast<void**>(&e->memory), slots * memory_ints * sizeof(int32_t));
  alloc(reinterpret_cast<void**>(&e->masks), slots * layout->words_padded * sizeof(uint32_t));
  alloc(reinterpret_cast<void**>(&e->base), slots * sizeof(uint32_t*));
  alloc(reinterpret_cast<void**>(&e->delta), slots * sizeof(uint32_t*));
  alloc(reinterpret_cast<void**>(&e->cursors), slots * sizeof(int32_t));
  alloc(reinterpret_cast<void**>(&e->active), slots * sizeof(int32_t));
  alloc(reinterpret_cast<void**>(&e->tokens), slots * sizeof(int32_t));
  alloc(reinterpret_cast<void**>(&e->faults), sizeof(int32_t));
  alloc(reinterpret_cast<void**>(&e->admissions), slots * sizeof(XgAdmission));
  if (err != cudaSuccess) {
    release(e);
    cudaGetLastError();
    return fail(XG_ENOMEM, std::string("device allocation failed: ") + cudaGetErrorString(err));
  }
  err = cudaMemcpy(e->blob, blob, static_cast<size_t>(layout->blob_bytes),
                   on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice);
  if (err == cudaSuccess) err = cudaMemset(e->memory, 0, slots * memory_ints * sizeof(int32_t));
  if (err == cudaSuccess) err = cudaMemset(e->masks, 0, slots * layout->words_padded * sizeof(uint32_t));
  if (err == cudaSuccess) err = cudaMemset(e->faults, 0, sizeof(int32_t));
  if (err != cudaSuccess) {
    release(e);
    return cuda_fail(err, "engine upload");
  }
  bind_tables(e);
  if (int rc = load_blob_versions(e, on_device ? nullptr : blob)) {
    release(e);
    return rc;
  }
  // one mask row; with release on, then the mass passes' ring (kRingBytes per thread)
  e->composed_bytes = static_cast<size_t>(layout->words_padded) * sizeof(uint32_t) +
                      (e->t.release_on ? static_cast<size_t>(kFusedThreads) * kRingBytes : 0);
  for (const void* kernel : {reinterpret_cast<const void*>(sync_apply_kernel<4>),
                             reinterpret_cast<const void*>(sync_apply_kernel<2>),
                             reinterpret_cast<const void*>(draft_apply_kernel<4>),
                             reinterpret_cast<const void*>(draft_apply_kernel<2>)}) {
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(e->composed_bytes));
    if (err != cudaSuccess) {
      release(e);
      return cuda_fail(err, "sync_apply shared memory (vocabulary too large for one mask row on chip)");
    }
  }
  {
    const void* host = on_device ? nullptr : blob;
    int rc = fill_delimiter_offsets(e->t.closer, e->blob, layout->closer_off, host);
    if (!rc) rc = fill_delimiter_offsets(e->t.separator, e->blob, layout->separator_off, host);
    if (!rc) rc = fill_delimiter_offsets(e->t.escape, e->blob, layout->escape_off, host);
    if (rc) {
      release(e);
      return rc;
    }
  }
  if (int rc = derive_tables(e)) {
    release(e);
    return rc;
  }
  begin_kernel<<<static_cast<unsigned>((slots + 127) / 128), 128>>>(e->t, nullptr, max_sequences, 0, max_sequences);
  err = cudaGetLastError();
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  if (err != cudaSuccess) {
    release(e);
    return cuda_fail(err, "engine initialization");
  }
  *out = e;
  return XG_OK;
}

// The derived write-planning tables (derive_kernel), once per engine.
int derive_tables(XgEngine* e) {
  const int32_t wp = e->layout.words_padded, vocab = e->layout.vocab;
  cudaError_t err = cudaMalloc(reinterpret_cast<void**>(&e->rel_any), static_cast<size_t>(wp) * sizeof(uint32_t));
  if (err == cudaSuccess)
    err = cudaMalloc(reinterpret_cast<void**>(&e->rel_any_tok), static_cast<size_t>(vocab > 0 ? vocab : 1) * sizeof(int32_t));
  if (err == cudaSuccess) err = cudaMalloc(reinterpret_cast<void**>(&e->sparse), 64 * (1 + kSparseBlocked) * sizeof(int32_t));
  if (err != cudaSuccess) {
    cudaGetLastError();
    return fail(XG_ENOMEM, std::string("device allocation failed: ") + cudaGetErrorString(err));
  }
  int32_t* scratch = nullptr;  // the kernel's three results
  err = cudaMalloc(reinterpret_cast<void**>(&scratch), 3 * sizeof(int32_t));
  if (err == cudaSuccess) err = cudaMemset(scratch, 0, 3 * sizeof(int32_t));
  if (err == cudaSuccess) err = cudaMemset(e->rel_any, 0, static_cast<size_t>(wp) * sizeof(uint32_t));
  if (err == cudaSuccess) {
    derive_kernel<<<1, 1024>>>(e->t, e->rel_any, e->rel_any_tok, e->sparse, scratch, e->layout.opener_len,
                               e->layout.closer_len);
    err = cudaGetLastError();
  }
  int32_t host[3] = {0, 0, 0};
  if (err == cudaSuccess) err = cudaMemcpy(host, scratch, sizeof(host), cudaMemcpyDeviceToHost);
  cudaFree(scratch);
  if (err != cudaSuccess) return cuda_fail(err, "engine set-up (derived tables)");
  e->t.rel_any = e->rel_any;
  e->t.rel_any_tok = e->rel_any_tok;
  e->t.rel_any_count = host[0];
  e->t.sparse = e->sparse;
  e->t.free_sparse = static_cast<uint32_t>(host[1]);
  e->t.esc_sparse = static_cast<uint32_t>(host[2]);
  return XG_OK;
}

int check_slot(const XgEngine* e, int32_t slot) {
  if (slot < 0 || slot >= e->max_sequences)
    return fail(XG_EINVAL, "slot must be between 0 and max_sequences - 1, got " + std::to_string(slot));
  return XG_OK;
}

int slot_op(XgEngine* e, const SlotArgs& a, void* stream) {
  slot_kernel<<<1, 32, 0, as_stream(stream)>>>(e->t, a);
  XG_CUDA(cudaGetLastError(), "slot kernel");
  return XG_OK;
}

int launch_step(XgEngine* e, const StepArgs& a, void* stream) {
  if (a.count == 0) return XG_OK;
  step_kernel<<<static_cast<unsigned>((a.count + kWarpsPerBlock - 1) / kWarpsPerBlock), kWarpsPerBlock * 32, 0,
                as_stream(stream)>>>(e->t, a);
  XG_CUDA(cudaGetLastError(), "step kernel");
  return XG_OK;
}

char* data_of(void* logits) { return static_cast<char*>(logits); }

// g_noalloc_scratch's device address, looked up once per device (with that device current).
constexpr int kNoAllocDevices = 64;
std::mutex g_noalloc_lock;
char* g_noalloc_address[kNoAllocDevices] = {};

int noalloc_scratch(int device, char** out) {
  if (device < 0 || device >= kNoAllocDevices) return fail(XG_EINVAL, "device ordinal out of range");
  std::lock_guard<std::mutex> hold(g_noalloc_lock);
  if (g_noalloc_address[device] == nullptr) {
    void* address = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&address, g_noalloc_scratch);
    if (err != cudaSuccess || address == nullptr) {
      cudaGetLastError();
      return fail(XG_ECUDA, std::string("static draft scratch: cudaGetSymbolAddress failed: ") +
                                cudaGetErrorString(err));
    }
    g_noalloc_address[device] = static_cast<char*>(address);
  }
  *out = g_noalloc_address[device];
  return XG_OK;
}

// Launch the row kernel: draft rows with scratch for `rows` rows at `scratch` (memory rows
// first), or, without local_pos, every row at its slot's own state (no scratch).
int launch_drafts(XgEngine* e, char* logits, int32_t dtype, int32_t rows, int32_t cols, int64_t row_stride,
                  const int32_t* row_slots, const int32_t* local_pos, const int32_t* input_ids, char* scratch,
                  void* stream) {
  DraftArgs d{};
  d.row_slots = row_slots;
  d.local_pos = local_pos;
  d.input_ids = input_ids;
  d.max_slots = e->max_sequences;
  if (scratch) {
    d.scratch_memory = reinterpret_cast<int32_t*>(scratch);
    d.scratch_masks = reinterpret_cast<uint32_t*>(scratch + static_cast<int64_t>(rows) * e->t.memory_ints * 4);
  }
  cudaStream_t s = as_stream(stream);
  const size_t released = e->t.release_on ? e->composed_bytes : 0;  // a released row's mask and the ring
  if (dtype == XG_F32)
    draft_apply_kernel<4><<<rows, kFusedThreads, released, s>>>(e->t, d, logits, cols, row_stride, 0xff800000u);
  else
    draft_apply_kernel<2><<<rows, kFusedThreads, released, s>>>(e->t, d, logits, cols, row_stride,
                                                                 dtype == XG_BF16 ? 0xff80u : 0xfc00u);
  XG_CUDA(cudaGetLastError(), "draft apply kernel");
  return XG_OK;
}

// Host admissions are checked, then copied into the engine's staging buffer on `stream`;
// device admissions are used in place (the kernels skip and count entries out of range).
int stage_admissions(XgEngine* e, const XgAdmission* admissions, int32_t count, int32_t on_host, void* stream,
                     const XgAdmission** out) {
  *out = nullptr;
  if (count < 0 || count > e->max_sequences)
    return fail(XG_EINVAL, "admissions must number between 0 and max_sequences (" + std::to_string(e->max_sequences) +
                               "), got " + std::to_string(count));
  if (count == 0) return XG_OK;
  if (!admissions) return fail(XG_EINVAL, "null admissions");
  if (!on_host) {
    *out = admissions;
    return XG_OK;
  }
  for (int32_t j = 0; j < count; ++j) {
    const XgAdmission& a = admissions[j];
    if (int rc = check_slot(e, a.slot)) return rc;
    for (int32_t k = 0; k < j; ++k)
      if (admissions[k].slot == a.slot) return fail(XG_EINVAL, "two admissions name slot " + std::to_string(a.slot));
    if (a.on != 0 && a.on != 1) return fail(XG_EINVAL, "admission `on` must be 0 or 1");
    if (a.version < 0 || a.version > e->t.versions || (a.version > 0 && !e->arena.versions[a.version - 1].live))
      return fail(XG_EINVAL, "KG version must be 0 or a registered version up to " + std::to_string(e->t.versions) + ", got " +
                                 std::to_string(a.version));
    if (a.anchor_count < 0 || a.anchor_count > XG_MAX_ANCHORS)
      return fail(XG_EINVAL, "an admission holds 0 to 64 anchor rows");
    for (int32_t k = 0; k < a.anchor_count; ++k)
      if (a.anchors[k] < 0 || a.anchors[k] >= e->layout.entity_rows || (k > 0 && a.anchors[k] <= a.anchors[k - 1]))
        return fail(XG_EINVAL, "anchor rows must be sorted, distinct label rows of the index");
  }
  XG_CUDA(cudaMemcpyAsync(e->admissions, admissions, count * sizeof(XgAdmission), cudaMemcpyHostToDevice,
                          as_stream(stream)),
          "admission upload");
  *out = e->admissions;
  return XG_OK;
}

int launch_admit(XgEngine* e, const XgAdmission* admit, int32_t count, void* stream) {
  admit_kernel<<<count, 32, 0, as_stream(stream)>>>(e->t, admit, e->max_sequences, e->faults);
  XG_CUDA(cudaGetLastError(), "admit kernel");
  return XG_OK;
}

int copy_host(void* out, const void* device, size_t bytes) {
  XG_CUDA(cudaDeviceSynchronize(), "engine step");
  if (bytes) XG_CUDA(cudaMemcpy(out, device, bytes, cudaMemcpyDeviceToHost), "copy to host");
  return XG_OK;
}

}  // namespace

extern "C" {

const char* xg_last_error(void) { return g_error.c_str(); }

int32_t xg_abi_version(void) { return XG_ABI_VERSION; }

int xg_create(const void* blob_host, const XgLayout* layout, const XgOptions* options, int32_t max_sequences,
              XgEngine** out) {
  return create(blob_host, false, layout, options, max_sequences, out);
}

int xg_create_from_device(const void* blob_device, const XgLayout* layout, const XgOptions* options,
                          int32_t max_sequences, XgEngine** out) {
  return create(blob_device, true, layout, options, max_sequences, out);
}

int xg_destroy(XgEngine* engine) {
  if (!engine) return XG_OK;
  cudaDeviceSynchronize();
  release(engine);
  return XG_OK;
}

int xg_info(const XgEngine* e, XgInfo* out) {
  if (!e || !out) return fail(XG_EINVAL, "null argument");
  *out = XgInfo{e->max_sequences, e->layout.vocab, e->layout.words, e->layout.words_padded, e->t.memory_ints, e->device};
  return XG_OK;
}

int xg_reset(XgEngine* e, void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  begin_kernel<<<static_cast<unsigned>((e->max_sequences + 127) / 128), 128, 0, as_stream(stream)>>>(
      e->t, nullptr, e->max_sequences, 0, e->max_sequences);
  XG_CUDA(cudaGetLastError(), "reset kernel");
  return XG_OK;
}

int xg_begin(XgEngine* e, const int32_t* slots, int32_t count, int32_t on, void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  if (count < 0 || count > e->max_sequences) return fail(XG_EINVAL, "more slots than max_sequences");
  if (count == 0) return XG_OK;
  if (!slots) return fail(XG_EINVAL, "null slots");
  begin_kernel<<<static_cast<unsigned>((count + 127) / 128), 128, 0, as_stream(stream)>>>(e->t, slots, count, on ? 1 : 0,
                                                                                          e->max_sequences);
  XG_CUDA(cudaGetLastError(), "begin kernel");
  return XG_OK;
}

int xg_set_reached(XgEngine* e, int32_t slot, const int32_t* rows, int32_t count, void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  if (int rc = check_slot(e, slot)) return rc;
  if (count <= 0 || !rows) return fail(XG_EINVAL, "anchor has no writable label rows");
  SlotArgs a{};
  a.slot = slot;
  a.op = 2;
  a.count = count < kMaxSet ? count : kMaxSet;
  for (int32_t i = 0; i < a.count; ++i) {
    if (rows[i] < 0 || rows[i] >= e->layout.entity_rows || (i > 0 && rows[i] <= rows[i - 1]))
      return fail(XG_EINVAL, "anchor rows must be sorted, distinct label rows of the index");
    a.rows[i] = rows[i];
  }
  return slot_op(e, a, stream);
}

int xg_set_version(XgEngine* e, int32_t slot, int32_t version, void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  if (int rc = check_slot(e, slot)) return rc;
  if (version < 0 || version > e->t.versions || (version > 0 && !e->arena.versions[version - 1].live))
    return fail(XG_EINVAL, "KG version must be 0 or a registered version up to " + std::to_string(e->t.versions) + ", got " +
                               std::to_string(version));
  SlotArgs a{};
  a.slot = slot;
  a.op = 1;
  a.value = version;
  return slot_op(e, a, stream);
}

int xg_open_span(XgEngine* e, int32_t slot, void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  if (int rc = check_slot(e, slot)) return rc;
  SlotArgs a{};
  a.slot = slot;
  a.op = 0;
  return slot_op(e, a, stream);
}

int xg_enable_stop(XgEngine* e, const int64_t* label_offsets, const uint8_t* label_words, int64_t word_bytes) {
  if (!e || !label_offsets || (word_bytes > 0 && !label_words)) return fail(XG_EINVAL, "null argument");
  if (!e->t.paths || !e->t.committed) return fail(XG_EINVAL, "residual-goal STOP needs committed paths (committed_paths=True)");
  if (e->stop_on) return fail(XG_EINVAL, "STOP is already enabled on this engine");
  if (e->t.relation_mode != 0) return fail(XG_EINVAL, "weaker relations need path mode without STOP");
  const int64_t rows = e->layout.entity_rows;
  if (label_offsets[0] != 0 || label_offsets[rows] != word_bytes)
    return fail(XG_EINVAL, "STOP label words: offsets must run from 0 to the word bytes, one row per label row");
  for (int64_t r = 0; r < rows; ++r)
    if (label_offsets[r + 1] < label_offsets[r]) return fail(XG_EINVAL, "STOP label word offsets must not decrease");
  const int64_t slots = e->max_sequences;
  cudaError_t err = cudaSuccess;
  auto alloc = [&](void** p, size_t bytes) {
    if (err == cudaSuccess) err = cudaMalloc(p, bytes > 0 ? bytes : 16);
  };
  alloc(reinterpret_cast<void**>(&e->stop_label_off), (rows + 1) * sizeof(int64_t));
  alloc(reinterpret_cast<void**>(&e->stop_label_words), static_cast<size_t>(word_bytes));
  alloc(reinterpret_cast<void**>(&e->stop_on), slots * sizeof(int32_t));
  alloc(reinterpret_cast<void**>(&e->stop_rel), slots * static_cast<size_t>(e->t.relations) * 3 * sizeof(int32_t));
  alloc(reinterpret_cast<void**>(&e->stop_woff), slots * (kMaxStopWords + 2) * sizeof(int32_t));
  alloc(reinterpret_cast<void**>(&e->stop_words), slots * static_cast<size_t>(kMaxStopBytes));
  if (err == cudaSuccess)
    err = cudaMemcpy(e->stop_label_off, label_offsets, (rows + 1) * sizeof(int64_t), cudaMemcpyHostToDevice);
  if (err == cudaSuccess && word_bytes > 0)
    err = cudaMemcpy(e->stop_label_words, label_words, static_cast<size_t>(word_bytes), cudaMemcpyHostToDevice);
  if (err == cudaSuccess) err = cudaMemset(e->stop_on, 0, slots * sizeof(int32_t));
  if (err != cudaSuccess) {
    for (void* p : {static_cast<void*>(e->stop_label_off), static_cast<void*>(e->stop_label_words),
                    static_cast<void*>(e->stop_on), static_cast<void*>(e->stop_rel), static_cast<void*>(e->stop_woff),
                    static_cast<void*>(e->stop_words)})
      cudaFree(p);
    e->stop_label_off = nullptr;
    e->stop_label_words = nullptr;
    e->stop_on = e->stop_rel = e->stop_woff = nullptr;
    e->stop_words = nullptr;
    return cuda_fail(err, "STOP tables");
  }
  e->t.stop_label_off = e->stop_label_off;
  e->t.stop_label_words = e->stop_label_words;
  e->t.stop_on = e->stop_on;
  e->t.stop_rel = e->stop_rel;
  e->t.stop_woff = e->stop_woff;
  e->t.stop_words = e->stop_words;
  return XG_OK;
}

int xg_set_stop(XgEngine* e, int32_t slot, const int32_t* relations, int32_t relation_count, const uint8_t* words,
                int32_t word_bytes, const int32_t* offsets, int32_t offset_count, void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  if (!e->stop_on) return fail(XG_EINVAL, "STOP is not enabled (stop='residual-goal')");
  if (int rc = check_slot(e, slot)) return rc;
  if (!relations || !offsets || (word_bytes > 0 && !words)) return fail(XG_EINVAL, "null argument");
  const int32_t count = offset_count - 1;
  if (relation_count != e->t.relations || count < 0 || count > kMaxStopWords || word_bytes < 0 ||
      word_bytes > kMaxStopBytes)
    return fail(XG_EINVAL, "STOP needs one entry per relation and at most 64 question words of 4096 bytes");
  if (offsets[0] != 0 || offsets[count] != word_bytes)
    return fail(XG_EINVAL, "STOP word offsets must cover the word bytes");
  for (int32_t k = 0; k < count; ++k)
    if (offsets[k + 1] < offsets[k]) return fail(XG_EINVAL, "STOP word offsets must not decrease");
  std::vector<int32_t> woff(kMaxStopWords + 2, 0);
  woff[0] = count;
  for (int32_t k = 0; k <= count; ++k) woff[k + 1] = offsets[k];
  cudaStream_t s = as_stream(stream);
  static const int32_t on = 1;
  XG_CUDA(cudaMemcpyAsync(e->stop_rel + static_cast<int64_t>(slot) * e->t.relations * 3, relations,
                          static_cast<size_t>(relation_count) * 3 * sizeof(int32_t), cudaMemcpyHostToDevice, s),
          "STOP upload");
  XG_CUDA(cudaMemcpyAsync(e->stop_woff + static_cast<int64_t>(slot) * (kMaxStopWords + 2), woff.data(),
                          woff.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s),
          "STOP upload");
  if (word_bytes > 0)
    XG_CUDA(cudaMemcpyAsync(e->stop_words + static_cast<int64_t>(slot) * kMaxStopBytes, words,
                            static_cast<size_t>(word_bytes), cudaMemcpyHostToDevice, s),
            "STOP upload");
  XG_CUDA(cudaMemcpyAsync(e->stop_on + slot, &on, sizeof(int32_t), cudaMemcpyHostToDevice, s), "STOP upload");
  // the staging vector is pageable: the copies above have read it when they return
  return XG_OK;
}

int xg_advance(XgEngine* e, const int32_t* tokens, int32_t count, int32_t tokens_on_host, void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  if (count < 0 || count > e->max_sequences)
    return fail(XG_EINVAL, "sequences must be between 0 and max_sequences (" + std::to_string(e->max_sequences) +
                               "), got " + std::to_string(count));
  if (count == 0) return XG_OK;
  if (!tokens) return fail(XG_EINVAL, "null tokens");
  const int32_t* device_tokens = tokens;
  if (tokens_on_host) {
    XG_CUDA(cudaMemcpyAsync(e->tokens, tokens, count * sizeof(int32_t), cudaMemcpyHostToDevice, as_stream(stream)),
            "token upload");
    device_tokens = e->tokens;
  }
  StepArgs a{};
  a.tokens = device_tokens;
  a.count = count;
  return launch_step(e, a, stream);
}

int xg_sync(XgEngine* e, const int32_t* slots, int32_t count, const int32_t* history, int64_t history_stride,
            int64_t history_rows, const int32_t* prompt_len, const int32_t* total_len, int64_t lengths_count,
            void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  if (count < 0 || count > e->max_sequences) return fail(XG_EINVAL, "more slots than max_sequences");
  if (lengths_count < e->max_sequences) return fail(XG_EINVAL, "prompt_len and total_len need one entry per slot");
  if (history_rows < e->max_sequences || history_stride < 0)
    return fail(XG_EINVAL, "history needs one contiguous row per slot");
  if (count == 0) return XG_OK;
  if (!slots || !history || !prompt_len || !total_len) return fail(XG_EINVAL, "null argument");
  StepArgs a{};
  a.slots = slots;
  a.history = history;
  a.stride = history_stride;
  a.prompt_len = prompt_len;
  a.total_len = total_len;
  a.count = count;
  return launch_step(e, a, stream);
}

int xg_fill_mask(XgEngine* e, int32_t sequences, void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  if (sequences < 0 || sequences > e->max_sequences)
    return fail(XG_EINVAL, "sequences must be between 0 and max_sequences (" + std::to_string(e->max_sequences) +
                               "), got " + std::to_string(sequences));
  if (sequences == 0) return XG_OK;
  fill_kernel<<<sequences, 256, 0, as_stream(stream)>>>(e->t);
  XG_CUDA(cudaGetLastError(), "fill kernel");
  return XG_OK;
}

int xg_mask_device(XgEngine* e, uint32_t** out) {
  if (!e || !out) return fail(XG_EINVAL, "null argument");
  *out = e->masks;
  return XG_OK;
}

int xg_states_device(XgEngine* e, XgState** out) {
  if (!e || !out) return fail(XG_EINVAL, "null argument");
  *out = e->states;
  return XG_OK;
}

int xg_mask_host(XgEngine* e, int32_t sequences, uint32_t* out) {
  if (!e || (!out && sequences)) return fail(XG_EINVAL, "null argument");
  if (sequences < 0 || sequences > e->max_sequences) return fail(XG_EINVAL, "sequences out of range");
  XG_CUDA(cudaDeviceSynchronize(), "engine step");
  if (sequences == 0) return XG_OK;
  XG_CUDA(cudaMemcpy2D(out, e->layout.words * sizeof(uint32_t), e->masks, e->layout.words_padded * sizeof(uint32_t),
                       e->layout.words * sizeof(uint32_t), sequences, cudaMemcpyDeviceToHost),
          "copy to host");
  return XG_OK;
}

int xg_states_host(XgEngine* e, int32_t sequences, int32_t* out) {
  if (!e || (!out && sequences)) return fail(XG_EINVAL, "null argument");
  if (sequences < 0 || sequences > e->max_sequences) return fail(XG_EINVAL, "sequences out of range");
  return copy_host(out, e->states, static_cast<size_t>(sequences) * sizeof(XgState));
}

int xg_memory_host(XgEngine* e, int32_t sequences, int32_t* out) {
  if (!e || (!out && sequences)) return fail(XG_EINVAL, "null argument");
  if (sequences < 0 || sequences > e->max_sequences) return fail(XG_EINVAL, "sequences out of range");
  return copy_host(out, e->memory, static_cast<size_t>(sequences) * e->t.memory_ints * sizeof(int32_t));
}

int xg_sync_apply(XgEngine* e, const int32_t* slots, int32_t count, const int32_t* history, int64_t history_stride,
                  int64_t history_rows, const int32_t* prompt_len, const int32_t* total_len, int64_t lengths_count,
                  void* logits, int32_t dtype, int32_t cols, int64_t row_stride, void* stream) {
  return xg_sync_apply_admit(e, slots, count, history, history_stride, history_rows, prompt_len, total_len,
                             lengths_count, logits, dtype, cols, row_stride, nullptr, 0, 0, stream);
}

int xg_sync_apply_admit(XgEngine* e, const int32_t* slots, int32_t count, const int32_t* history,
                        int64_t history_stride, int64_t history_rows, const int32_t* prompt_len,
                        const int32_t* total_len, int64_t lengths_count, void* logits, int32_t dtype, int32_t cols,
                        int64_t row_stride, const XgAdmission* admissions, int32_t admit_count,
                        int32_t admissions_on_host, void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  if (count < 0 || count > e->max_sequences) return fail(XG_EINVAL, "more slots than max_sequences");
  if (lengths_count < e->max_sequences) return fail(XG_EINVAL, "prompt_len and total_len need one entry per slot");
  if (history_rows < e->max_sequences || history_stride < 0)
    return fail(XG_EINVAL, "history needs one contiguous row per slot");
  if (cols < 0 || row_stride < cols) return fail(XG_EINVAL, "logits need one contiguous row per slot");
  if (dtype != XG_F32 && dtype != XG_BF16 && dtype != XG_F16) return fail(XG_EINVAL, "logits must be float32, bfloat16 or float16");
  if (static_cast<int64_t>(count) * ((cols + 1023) / 1024) > 0x7fffffff) return fail(XG_EINVAL, "too many logits rows");
  const XgAdmission* admit = nullptr;
  if (int rc = stage_admissions(e, admissions, admit_count, admissions_on_host, stream, &admit)) return rc;
  if (count == 0) {
    if (admit_count == 0) return XG_OK;
    return launch_admit(e, admit, admit_count, stream);  // nothing to step: the admissions alone
  }
  if (!slots || !history || !prompt_len || !total_len || !logits) return fail(XG_EINVAL, "null argument");
  const int elt = dtype == XG_F32 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(logits) % elt) return fail(XG_EINVAL, "logits are not aligned to their element size");
  FusedArgs f{};
  f.a.slots = slots;
  f.a.history = history;
  f.a.stride = history_stride;
  f.a.prompt_len = prompt_len;
  f.a.total_len = total_len;
  f.a.count = count;
  f.admit = admit;
  f.admit_count = admit_count;
  f.max_slots = e->max_sequences;
  f.logits = static_cast<char*>(logits);
  f.stride = row_stride;
  f.cols = cols;
  f.neg = dtype == XG_F32 ? 0xff800000u : dtype == XG_BF16 ? 0xff80u : 0xfc00u;
  f.faults = e->faults;
  cudaStream_t s = as_stream(stream);
  if (elt == 4)
    sync_apply_kernel<4><<<count, kFusedThreads, e->composed_bytes, s>>>(e->t, f);
  else
    sync_apply_kernel<2><<<count, kFusedThreads, e->composed_bytes, s>>>(e->t, f);
  XG_CUDA(cudaGetLastError(), "sync_apply kernel");
  return XG_OK;
}

int xg_admit(XgEngine* e, const XgAdmission* admissions, int32_t count, int32_t on_host, void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  const XgAdmission* admit = nullptr;
  if (int rc = stage_admissions(e, admissions, count, on_host, stream, &admit)) return rc;
  if (count == 0) return XG_OK;
  return launch_admit(e, admit, count, stream);
}

int xg_add_version(XgEngine* e, const int32_t* subjects, int32_t count, const int64_t* adjacency,
                   const int32_t* edge_relations, const int32_t* edge_objects, void* stream, int32_t* version) {
  if (!e || !version) return fail(XG_EINVAL, "null argument");
  if (e->t.relation_mode == 2)
    return fail(XG_EINVAL, "successor support reads the successor tables of the versions built in; "
                           "no version can be added while it runs");
  return add_version(e, subjects, count, adjacency, edge_relations, edge_objects, as_stream(stream), version);
}

int xg_set_relation_successors(XgEngine* e, const uint32_t* tables, int32_t table_count) {
  if (!e || !tables) return fail(XG_EINVAL, "null argument");
  if (e->t.relation_mode != 2) return fail(XG_EINVAL, "successor tables need relations = 2 (successor)");
  if (table_count < 1 + e->layout.versions)
    return fail(XG_EINVAL, "successor support needs one table for the base KG and one per built-in version");
  const size_t bytes = static_cast<size_t>(table_count) * e->t.relations * e->t.relation_words * sizeof(uint32_t);
  uint32_t* device = nullptr;
  cudaError_t err = cudaMalloc(reinterpret_cast<void**>(&device), bytes > 0 ? bytes : 16);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return fail(XG_ENOMEM, std::string("device allocation failed: ") + cudaGetErrorString(err));
  }
  if (bytes > 0) err = cudaMemcpy(device, tables, bytes, cudaMemcpyHostToDevice);
  if (err != cudaSuccess) {
    cudaFree(device);
    return cuda_fail(err, "successor tables upload");
  }
  cudaFree(e->successors);  // (the engine's stream is idle: the copy above synchronized)
  e->successors = device;
  e->successor_tables = table_count;
  e->t.successors = device;
  e->t.successor_tables = table_count;
  return XG_OK;
}

int xg_set_expressions(XgEngine* e, const int32_t* delimiters, int64_t delimiter_ints, int32_t operators,
                       const int32_t* operator_lcp, const int32_t* date_entities, const int32_t* date_keys,
                       int32_t dates, const int32_t* verdicts) {
  if (!e || !delimiters || !operator_lcp || (dates > 0 && (!date_entities || !date_keys)))
    return fail(XG_EINVAL, "null argument");
  if (!e->options.expressions) return fail(XG_EINVAL, "expression tables need an engine created with expressions = 1");
  if (operators < 1 || operators > kMaxOperators)
    return fail(XG_EINVAL, "expressions offer 1 to 4 operators");
  if (operators > 2 && !verdicts) return fail(XG_EINVAL, "a value comparison needs the verdict entities, yes and no");
  if (dates < 0 || delimiter_ints < 1) return fail(XG_EINVAL, "negative table size");
  PackedDelim parsed[1 + kMaxOperators];
  if (!parse_packed_delims(delimiters, delimiter_ints, 1 + operators, e->layout.vocab, parsed))
    return fail(XG_EINVAL, "malformed expression delimiter lists");
  for (int32_t k = 0; k < operators * operators; ++k)
    if (operator_lcp[k] < 0 || operator_lcp[k] > 64) return fail(XG_EINVAL, "operator_lcp out of range");
  for (int32_t i = 0; i < dates; ++i) {
    if (date_entities[i] < 0 || date_entities[i] >= e->layout.entities || (i > 0 && date_entities[i] <= date_entities[i - 1]))
      return fail(XG_EINVAL, "date entities must be ascending entity positions");
  }
  if (verdicts) {
    for (int32_t k = 0; k < 2; ++k)
      if (verdicts[k] < 0 || verdicts[k] >= e->layout.entities) return fail(XG_EINVAL, "verdict entity out of range");
  }
  std::vector<int32_t> host(static_cast<size_t>(delimiter_ints) + 4 * static_cast<size_t>(dates));
  std::memcpy(host.data(), delimiters, delimiter_ints * sizeof(int32_t));
  int32_t* table = host.data() + delimiter_ints;
  for (int32_t i = 0; i < dates; ++i) {
    table[i] = date_entities[i];
    table[dates + i] = date_keys[i];
    table[2 * dates + i] = date_bound(date_keys[i], true);
    table[3 * dates + i] = date_bound(date_keys[i], false);
  }
  int32_t* device = nullptr;
  cudaError_t err = cudaMalloc(reinterpret_cast<void**>(&device), host.size() * sizeof(int32_t));
  if (err != cudaSuccess) {
    cudaGetLastError();
    return fail(XG_ENOMEM, std::string("device allocation failed: ") + cudaGetErrorString(err));
  }
  err = cudaMemcpy(device, host.data(), host.size() * sizeof(int32_t), cudaMemcpyHostToDevice);
  if (err != cudaSuccess) {
    cudaFree(device);
    return cuda_fail(err, "expression tables upload");
  }
  cudaFree(e->expr);  // (the engine's stream is idle: the copy above synchronized)
  e->expr = device;
  e->expr_delim_ints = delimiter_ints;
  e->operator_count = operators;
  for (int32_t k = 0; k < kMaxOperators * kMaxOperators; ++k) e->operator_lcp[k] = 0;
  for (int32_t k = 0; k < operators; ++k)
    for (int32_t j = 0; j < operators; ++j) e->operator_lcp[k * kMaxOperators + j] = operator_lcp[k * operators + j];
  for (int32_t k = 0; k <= operators; ++k) {
    Delim& d = k == 0 ? e->operand_sep : e->operators[k - 1];
    d = Delim{device + parsed[k].off, device + parsed[k].tok, device + parsed[k].next, parsed[k].len, {}};
    for (int32_t i = 0; i < 17; ++i) d.at[i] = parsed[k].at[i];
  }
  e->date_count = dates;
  e->verdict_yes = verdicts ? verdicts[0] : -1;
  e->verdict_no = verdicts ? verdicts[1] : -1;
  bind_expressions(e);
  return XG_OK;
}

int xg_drop_version(XgEngine* e, int32_t version, void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  VersionArena& a = e->arena;
  if (version < 1 || version > static_cast<int32_t>(a.versions.size()) || !a.versions[version - 1].live)
    return fail(XG_EINVAL, "no registered KG version " + std::to_string(version));
  static const int32_t empty[2] = {0, 0};
  XG_CUDA(cudaMemcpyAsync(a.range + 2 * (version - 1), empty, sizeof(empty), cudaMemcpyHostToDevice, as_stream(stream)),
          "version drop");
  a.versions[version - 1] = HostVersion{};
  return XG_OK;
}

int xg_faults(XgEngine* e, int32_t* out) {
  if (!e || !out) return fail(XG_EINVAL, "null argument");
  XG_CUDA(cudaDeviceSynchronize(), "engine step");
  XG_CUDA(cudaMemcpy(out, e->faults, sizeof(int32_t), cudaMemcpyDeviceToHost), "copy to host");
  XG_CUDA(cudaMemset(e->faults, 0, sizeof(int32_t)), "fault reset");
  return XG_OK;
}

int xg_apply_mask(XgEngine* e, void* logits, int32_t dtype, int32_t rows, int32_t cols, int64_t row_stride,
                  const int32_t* row_slots, const int32_t* local_pos, const int32_t* input_ids, void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  if ((local_pos == nullptr) != (input_ids == nullptr)) return fail(XG_EINVAL, "local_pos and input_ids go together");
  if (rows < 0 || cols < 0 || row_stride < cols) return fail(XG_EINVAL, "logits need one contiguous row per entry of row_slots");
  if (dtype != XG_F32 && dtype != XG_BF16 && dtype != XG_F16) return fail(XG_EINVAL, "logits must be float32, bfloat16 or float16");
  if (rows == 0 || cols == 0) return XG_OK;
  if (!logits || !row_slots) return fail(XG_EINVAL, "null argument");
  const int elt = dtype == XG_F32 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(logits) % elt) return fail(XG_EINVAL, "logits are not aligned to their element size");
  if (local_pos) {
    // draft rows: scratch for every row, grown (never shrunk) when a call has more rows
    // than any before it (the reference grows its row buffers the same way,
    // csrc/engine.cu:3006-3014)
    if (rows > e->draft_capacity) {
      XG_CUDA(cudaStreamSynchronize(as_stream(stream)), "draft scratch growth");
      cudaFree(e->draft_scratch);
      e->draft_scratch = nullptr;
      e->draft_capacity = 0;
      const cudaError_t err = cudaMalloc(&e->draft_scratch, static_cast<size_t>(rows) * draft_row_bytes(e->t));
      if (err != cudaSuccess) {
        e->draft_scratch = nullptr;
        cudaGetLastError();
        return fail(XG_ENOMEM, std::string("draft scratch allocation failed: ") + cudaGetErrorString(err));
      }
      e->draft_capacity = rows;
    }
    return launch_drafts(e, data_of(logits), dtype, rows, cols, row_stride, row_slots, local_pos, input_ids,
                         e->draft_scratch, stream);
  }
  // The logit policies need a whole row per CTA: the row kernel, every row at its slot's
  // own state (no drafts, no scratch).
  if (e->t.release_on || e->t.escape_bias != 0.0f)
    return launch_drafts(e, data_of(logits), dtype, rows, cols, row_stride, row_slots, nullptr, nullptr, nullptr,
                         stream);
  // Split each row into `chunks` CTAs so that the grid is about one wave of resident CTAs
  // (each CTA then runs long enough to hide its few dependent pointer loads).
  const int64_t per_row_max = ((static_cast<int64_t>(cols) + 1023) / 1024 + 7) / 8;  // >= 8 segments per CTA
  const int64_t wanted = (static_cast<int64_t>(e->sm_count) * kApplyCtasPerSm + rows - 1) / rows;
  const int32_t chunks = static_cast<int32_t>(wanted < 1 ? 1 : wanted > per_row_max ? (per_row_max < 1 ? 1 : per_row_max) : wanted);
  const int64_t blocks = static_cast<int64_t>(rows) * chunks;
  if (blocks > 0x7fffffff) return fail(XG_EINVAL, "too many logits rows");
  cudaLaunchConfig_t config{};
  config.gridDim = dim3(static_cast<unsigned>(blocks));
  config.blockDim = dim3(kApplyThreads);
  config.stream = as_stream(stream);
  cudaLaunchAttribute attribute{};
  attribute.id = cudaLaunchAttributeProgrammaticStreamSerialization;  // overlap our launch with the step kernel
  attribute.val.programmaticStreamSerializationAllowed = 1;
  config.attrs = &attribute;
  config.numAttrs = 1;
  char* data = static_cast<char*>(logits);
  if (dtype == XG_F32) {
    XG_CUDA(cudaLaunchKernelEx(&config, apply_kernel<4>, e->t, data, cols, row_stride, row_slots, chunks,
                               e->max_sequences, 0xff800000u),
            "apply kernel");
  } else {
    XG_CUDA(cudaLaunchKernelEx(&config, apply_kernel<2>, e->t, data, cols, row_stride, row_slots, chunks,
                               e->max_sequences, dtype == XG_BF16 ? 0xff80u : 0xfc00u),
            "apply kernel");
  }
  return XG_OK;
}

int xg_apply_mask_noalloc(XgEngine* e, void* logits, int32_t dtype, int32_t rows, int32_t cols, int64_t row_stride,
                          const int32_t* row_slots, const int32_t* local_pos, const int32_t* input_ids,
                          void* stream) {
  if (!e) return fail(XG_EINVAL, "null engine");
  if (!local_pos || !input_ids)
    return fail(XG_EINVAL, "xg_apply_mask_noalloc masks draft rows: local_pos and input_ids are required");
  if (rows < 0 || cols < 0 || row_stride < cols) return fail(XG_EINVAL, "logits need one contiguous row per entry of row_slots");
  if (dtype != XG_F32 && dtype != XG_BF16 && dtype != XG_F16) return fail(XG_EINVAL, "logits must be float32, bfloat16 or float16");
  const int64_t per_row = draft_row_bytes(e->t);
  if (static_cast<int64_t>(rows) * per_row > kNoAllocScratchBytes)
    return fail(XG_EINVAL, std::to_string(rows) + " draft rows need " + std::to_string(rows * per_row) +
                               " bytes of scratch; xg_apply_mask_noalloc has " + std::to_string(kNoAllocScratchBytes) +
                               " (at most " + std::to_string(kNoAllocScratchBytes / per_row) +
                               " rows with this vocabulary); use xg_apply_mask");
  if (rows == 0 || cols == 0) return XG_OK;
  if (!logits || !row_slots) return fail(XG_EINVAL, "null argument");
  const int elt = dtype == XG_F32 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(logits) % elt) return fail(XG_EINVAL, "logits are not aligned to their element size");
  int device = -1;
  XG_CUDA(cudaGetDevice(&device), "current device");
  if (device != e->device)
    return fail(XG_EINVAL, "call xg_apply_mask_noalloc with the engine's device current (device " +
                               std::to_string(e->device) + ", current " + std::to_string(device) + ")");
  char* scratch = nullptr;
  if (int rc = noalloc_scratch(device, &scratch)) return rc;
  return launch_drafts(e, data_of(logits), dtype, rows, cols, row_stride, row_slots, local_pos, input_ids, scratch,
                       stream);
}

}  // extern "C"
