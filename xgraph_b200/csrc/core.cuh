// Per-row constraint logic of the KG span engine: advance one token, build one mask.
//
// The semantics are those of the reference Oracle (src/xgraph/oracle.py:736-1922, the
// span language with ordinary, derivation and path modes, escapes, repeats, KG versions,
// anchors, unquoted starts, sitelink ranks and end-after-answer).  The data layout is
// this engine's own (tables.py packs it; layout.h declares it).
//
// One WARP owns one request row.  The scalar state machine runs redundantly in all 32
// lanes (uniform control flow, broadcast loads, lane 0 stores); loops over rows, edges
// and candidates are spread over the lanes with ballots.  The same source also compiles
// as plain C++ (XG_GPU == 0) where every "warp" loop runs sequentially: that build is a
// test seam only (tests check it against the oracle on the CPU), never a fallback.
#pragma once

#include <stdint.h>

#include "layout.h"

// XG_HD: small helpers, inlined.  XG_COLD: the rare, heavy transitions (closing a span,
// changing segment, frontiers, sorts) and the adjacency lookups they share, kept out of
// line so that the per-token path stays a few kilobytes of code: a decode step starts
// with its code out of the instruction caches and out of L2, and every jump to a code
// line not yet fetched costs a memory round trip (straight-line code streams in well).
// XG_SHARED: helpers of the per-token path (candidate tests, row bounds, flags), inlined
// into it.  Loops are kept rolled (#pragma unroll 1) except short scans whose loads must
// issue together.
#if defined(__CUDACC__)
#define XG_HD __device__ __forceinline__
#define XG_COLD __device__ __noinline__
#define XG_SHARED __device__ __forceinline__
#define XG_GPU 1
#else
#include <algorithm>
#define XG_HD inline
#define XG_COLD inline
#define XG_SHARED inline
#define XG_GPU 0
#endif

namespace xg {

constexpr int32_t kMaxSet = 64;       // MAX_FACTS == MAX_REACHED (src/xgraph/oracle.py:172-175)
constexpr int32_t kMaxHops = 8;       // MAX_PATH_RELATIONS (src/xgraph/oracle.py:177)
constexpr int32_t kTopCap = 256;      // per-warp candidate buffer of the top-64 selections
constexpr int32_t kItemBatch = 1;     // rounds of slice items whose loads are issued together
constexpr int32_t kLoadBatch = 4;     // warp_for_loaded: rounds whose loads are issued together
constexpr int32_t kScratchInts = 2 * kMaxSet + 2 + 2 * kMaxSet + kMaxSet;
constexpr int32_t kMaxStopWords = 64;    // MAX_STOP_WORDS (src/xgraph/stopping.py:45)
constexpr int32_t kMaxStopBytes = 4096;  // MAX_STOP_BYTES (src/xgraph/stopping.py:46)
constexpr int32_t kSparseBlocked = 64;   // blocked tokens an automaton row may list (Tables::sparse)
constexpr int32_t kMaxOperators = 4;     // expressions: the most operators a syntax may offer
constexpr int8_t kReject = -1;
constexpr int8_t kComplete = -2;

enum Phase : int32_t { kFree = 0, kSpan = 1, kEscaped = 2, kError = 3 };
enum Segment : int32_t { kSubject = 0, kRelation = 1, kObject = 2 };
// (kComparison a date or value comparison of expressions; kRelationPlan a path closed under
// a weaker relation support: its labels written, nothing executed)
enum Closed : int32_t { kNone = 0, kUnresolved = 1, kEntitySpan = 2, kFactSpan = 3, kPathSpan = 4, kComparison = 5,
                        kRelationPlan = 6 };
// Relation support of a path's relation segments (src/xgraph/relations.py:18): the entity
// frontier (paths executed), every relation, or the successors of the preceding label's.
enum RelationMode : int32_t { kFrontierSupport = 0, kVocabularySupport = 1, kSuccessorSupport = 2 };
enum Flag : int32_t { kMayClose = 1, kMaySep = 2, kMayEsc = 4, kStop = 8 };

// Slot memory (int32 words per slot): counts, then the fixed lists, then the bitmap of
// the relations the current subjects / frontier have.
enum MemoryField : int32_t {
  kMemFacts = 0,      // fact spans recorded (<= 64), for repeats=False
  kMemReached = 1,    // reached rows (<= 64); 0 = no binding yet
  kMemFrontier = 2,   // path frontier entities (<= 64)
  kMemVersion = 3,    // KG version the slot reads (0 = base)
  kMemPendingLo = 4,  // the next frontier cached for relation-label rows [lo, hi) (lo -1: none)
  kMemPendingHi = 5,
  kMemPendingCount = 6,
  kMemFactRows = 8,                           // 64 x (subject key, relation key, object key)
  kMemReachedRows = kMemFactRows + 3 * kMaxSet,  // 64 sorted label rows
  kMemFrontierEnt = kMemReachedRows + kMaxSet,   // 64 entities
  kMemFrontierRank = kMemFrontierEnt + kMaxSet,  // their start ranks
  kMemPendingRank = kMemFrontierRank + kMaxSet,  // cached next frontier: ranks
  kMemPendingFirst = kMemPendingRank + kMaxSet,  //   and first label rows
  kMemHave = kMemPendingFirst + kMaxSet,         // relation bitmap
};

// Expressions: a comparison's operand region of slot memory, at Tables::mem_operand (after
// the relation bitmap): operand B's frontier (entities, start ranks, count), each operand's
// ranked starts (the written label row of the start of rank k), operand A's best values of
// a value comparison (a label row or a date key, and whether it is a date), and operand B's
// relation bitmap.
enum OperandField : int32_t {
  kOpFrontEnt = 0,
  kOpFrontRank = kOpFrontEnt + kMaxSet,
  kOpStartsA = kOpFrontRank + kMaxSet,
  kOpStartsB = kOpStartsA + kMaxSet,
  kOpFrontCount = kOpStartsB + kMaxSet,
  kOpValues = kOpFrontCount + 4,
  kOpDated = kOpValues + kMaxSet,
  kOpHave = kOpDated + kMaxSet,  // + relation words (rounded up to 4)
};

// Slot memory ints: the fixed fields and the relation bitmap, and with expressions the
// operand region after them (its offset: the ints without it).
#if defined(__CUDACC__)
__host__ __device__
#endif
inline int32_t memory_ints_for(int32_t relation_words, bool expressions) {
  const int32_t words4 = (relation_words + 3) & ~3;
  return kMemHave + words4 + (expressions ? kOpHave + words4 : 0);
}

struct Key {
  uint64_t a;
  uint32_t b;
  uint32_t pad;
};
XG_HD bool key_less(const Key& x, const Key& y) { return x.a < y.a || (x.a == y.a && x.b < y.b); }
XG_HD bool key_eq(const Key& x, const Key& y) { return x.a == y.a && x.b == y.b; }
XG_HD Key max_key() { return Key{~0ull, ~0u, 0u}; }
XG_HD bool is_max(const Key& k) { return k.a == ~0ull && k.b == ~0u; }

struct Rows {
  const int32_t* tok;
  const int32_t* off;
  const int32_t* owner;
  int32_t count;
  const int32_t* col;    // [cols][count]: token at depth d, -1 past the row's end
  const int32_t* first;  // [vocab + 1]: first row whose first token is >= t
  int32_t cols;
};


// A span delimiter inside spans: per byte position p, the sorted tokens continuing it
// from p and where they end.  The CSR offsets of the first positions are also carried
// by value (`at`, kernel-parameter space) so the mask builder reads no offset from memory.
struct Delim {
  const int32_t* off;
  const int32_t* tok;
  const int32_t* next;
  int32_t len;
  int32_t at[17];  // off[0 .. min(len, 16)]
};

XG_HD int32_t delim_begin(const Delim& d, int32_t pos) { return pos < 17 ? d.at[pos] : d.off[pos]; }
XG_HD int32_t delim_end(const Delim& d, int32_t pos) { return pos + 1 < 17 ? d.at[pos + 1] : d.off[pos + 1]; }

// Device (or host-seam) view of the packed tables plus the per-slot buffers.
struct Tables {
  Rows ent, rel;
  const int32_t* ent_first_row;
  const int32_t* row_first;    // first label row of each label row's owner (one load, no owner hop)
  const int32_t* row_degree;   // base-KG degree of each label row's owner (one load, no owner hop)
  const int32_t* ent_rows_off;
  const int32_t* ent_rows;
  const int32_t* adj_off;
  const int32_t* edge_rel;
  const int32_t* edge_obj;
  const int32_t* run_off;     // [entities + 1]: each entity's relation runs (CSR)
  const int32_t* runs;        // [runs + 1][2]: (relation, first edge), closed by (INT32_MAX, edges)
  const int32_t* run_rel;     // [runs]: the relation of each run
  const int32_t* edge_first;  // [edges]: object's first label row, bit 31 = the object has no triples
  const int32_t* sitelinks;    // null unless the sitelink rank is on
  const int32_t* row_sitelinks;  // the same per label row (no owner hop); null unless the rank is on
  const int32_t* kept_prefix;  // null unless some rows are not unbound candidates
  const uint32_t* root_mask;
  const int64_t* wide_keys;
  const uint32_t* wide_masks;
  int32_t wide_count;
  const int8_t* free_next;
  const uint32_t* free_mask;
  const int8_t* esc_next;
  const uint32_t* esc_mask;
  const uint32_t* eos_mask;
  Delim closer, separator, escape;
  // Per token, the next byte position of every (delimiter, position) pair in one word:
  // 4 bits at 4 * (offset of the delimiter + position), 0 = the token does not continue
  // it (closer at offset 0, separator after it, escape after that).  Null when the
  // delimiters are too long for 16 nibbles; the CSR lists then serve.
  const uint64_t* dstep;
  // KG versions: version v (1..versions) owns the sorted edited subjects
  // ver_subj[ver_range[2v - 2] .. ver_range[2v - 1]); subject i's whole edge list is
  // ver_edge_*[ver_adj[i] .. ver_adj[i + 1]) (an empty range: v reads the base KG).
  const int32_t* ver_range;
  const int32_t* ver_subj;
  const int32_t* ver_adj;
  const int32_t* ver_edge_rel;
  const int32_t* ver_edge_obj;
  int32_t versions;
  int32_t vocab, words, words_padded, entities, relations, relation_words;
  int32_t escapes, repeats, derivation, paths, bound_escapes, committed, end_after_answer;
  // weaker relation supports (RelationMode; kFrontierSupport: paths executed as usual).
  // Successor support reads successors[v][r1] (relation_words words): bit r2 says that
  // some object of an r1 edge is the subject of an r2 edge in KG version v; versions from
  // successor_tables on read table 0 (the host registers no such version).
  int32_t relation_mode;
  const uint32_t* successors;
  int32_t successor_tables;
  // expressions (operator_count 0: off): the operators offered, each after the label prefix
  // (the third, the value comparison, only with the verdict entities), operator_lcp[k * 4 +
  // j] the leading bytes operators k and j share, and the operand separator; the date table
  // (the date entities' positions, sorted, with their keys and interval bounds, packed as
  // xgraph_b200.dates packs them); the verdict entities (yes, no); and the offset of each
  // slot's operand region in its memory.
  int32_t operator_count;
  int32_t operator_lcp[kMaxOperators * kMaxOperators];
  Delim operators[kMaxOperators];
  Delim operand_sep;
  const int32_t* date_entities;
  const int32_t* date_keys;
  const int32_t* date_lo;
  const int32_t* date_hi;
  int32_t date_count;
  int32_t verdict_yes, verdict_no;
  int32_t mem_operand;
  // apply_mask's logit policies (off: release_on 0, escape_bias 0): release a span row to
  // the escape marker when its log allowed mass is below release_log_mass, or (release_top)
  // when its own top token is disallowed; add escape_bias to the tokens that commit to it.
  float release_log_mass, escape_bias;
  int32_t release_top, release_on;
  // residual-goal STOP (null stop_on: not enabled): every entity label row's case-folded
  // words (CSR, each word followed by a 0 byte); per slot: whether a table is installed,
  // per relation number (answer-head flag, covered question words low, high), and the
  // relevant question words (count, then byte offsets; their bytes)
  const int64_t* stop_label_off;
  const uint8_t* stop_label_words;
  int32_t* stop_on;           // [slots]
  const int32_t* stop_rel;    // [slots][relations][3]
  const int32_t* stop_woff;   // [slots][kMaxStopWords + 2]
  const uint8_t* stop_words;  // [slots][kMaxStopBytes]
  // Derived once per engine from the tables above (the device engine's write planning; the
  // host seam leaves them empty): rel_any, a mask row holding every relation label token at
  // any depth and every token of the delimiter lists -- a superset of every mask a state
  // in a relation segment can have -- and its tokens; and, for the free-text (opener) and
  // escaped (closer) automaton rows that block few tokens, those tokens: bit p of
  // free_sparse / esc_sparse says that row p of free_mask / esc_mask has a list, at
  // sparse[(p or 32 + p) * (1 + kSparseBlocked)]: its count, then its tokens.
  const uint32_t* rel_any;     // [words_padded]
  const int32_t* rel_any_tok;  // [rel_any_count]
  int32_t rel_any_count;
  const int32_t* sparse;       // [64][1 + kSparseBlocked]
  uint32_t free_sparse, esc_sparse;
  // per-slot engine buffers
  XgState* states;
  int32_t* memory;
  int32_t memory_ints;
  uint32_t* masks;           // [slots, words_padded]: each slot's own mask bits
  // A slot's mask is base | delta: base a precomputed table row (free text, escaped span,
  // EOS only, root or wide label mask), delta the slot's own buffer row.  Both null: the
  // error phase (apply_mask leaves the row alone).
  const uint32_t** base;
  uint32_t** delta;
  int32_t* cursors;
  int32_t* active;
};

// ---------------------------------------------------------------------------------------
// Warp primitives.  On the host seam each becomes the obvious sequential loop.

struct Warp {
  int32_t lane;
  XG_HD bool leader() const { return lane == 0; }
};

XG_HD void warp_sync() {
#if XG_GPU
  __syncwarp();
#endif
}

// Whether f(i) holds for some i in [begin, end); begin/end must be warp-uniform.
template <class F>
XG_HD bool warp_any(const Warp& w, int32_t begin, int32_t end, F f) {
#if XG_GPU
  #pragma unroll 1
  for (int32_t base = begin; base < end; base += 32) {
    const int32_t i = base + w.lane;
    const bool hit = i < end && f(i);
    if (__any_sync(0xffffffffu, hit)) return true;
  }
  return false;
#else
  (void)w;
  #pragma unroll 1
  for (int32_t i = begin; i < end; ++i)
    if (f(i)) return true;
  return false;
#endif
}

// f(i) for every i in [begin, end), spread over the lanes (f must not need other lanes).
template <class F>
XG_HD void warp_for(const Warp& w, int32_t begin, int32_t end, F f) {
#if XG_GPU
  #pragma unroll 1
  for (int32_t i = begin + w.lane; i < end; i += 32) f(i);
  __syncwarp();
#else
  (void)w;
  #pragma unroll 1
  for (int32_t i = begin; i < end; ++i) f(i);
#endif
}

// The least key(i) over i in [begin, end) (max_key() when empty).
// warp_for over [begin, end) whose body is split into load(i), independent memory reads,
// and use(i, loaded): the loads of kLoadBatch rounds are issued together before their
// uses run, so a long range costs one memory round trip per kLoadBatch rounds while the
// loop's code stays short.
template <class L, class U>
XG_HD void warp_for_loaded(const Warp& w, int32_t begin, int32_t end, L load, U use) {
#if XG_GPU
#pragma unroll 1
  for (int32_t base = begin; base < end; base += 32 * kLoadBatch) {
    decltype(load(0)) v[kLoadBatch];
#pragma unroll
    for (int32_t b = 0; b < kLoadBatch; ++b) {
      const int32_t i = base + 32 * b + w.lane;
      if (i < end) v[b] = load(i);
    }
#pragma unroll
    for (int32_t b = 0; b < kLoadBatch; ++b) {
      const int32_t i = base + 32 * b + w.lane;
      if (i < end) use(i, v[b]);
    }
  }
#else
  (void)w;
#pragma unroll 1
  for (int32_t i = begin; i < end; ++i) use(i, load(i));
#endif
}

template <class F>
XG_HD Key warp_min(const Warp& w, int32_t begin, int32_t end, F key) {
  Key best = max_key();
#if XG_GPU
  #pragma unroll 1
  for (int32_t i = begin + w.lane; i < end; i += 32) {
    const Key k = key(i);
    if (key_less(k, best)) best = k;
  }
  #pragma unroll 1
  for (int32_t d = 16; d > 0; d >>= 1) {
    Key o;
    o.a = __shfl_xor_sync(0xffffffffu, best.a, d);
    o.b = __shfl_xor_sync(0xffffffffu, best.b, d);
    o.pad = 0;
    if (key_less(o, best)) best = o;
  }
#else
  (void)w;
  #pragma unroll 1
  for (int32_t i = begin; i < end; ++i) {
    const Key k = key(i);
    if (key_less(k, best)) best = k;
  }
#endif
  return best;
}

XG_HD void set_bit(uint32_t* words, int32_t token) {
#if XG_GPU
  atomicOr(&words[token >> 5], 1u << (token & 31));
#else
  words[token >> 5] |= 1u << (token & 31);
#endif
}

// ---------------------------------------------------------------------------------------
// Top-64 selection over a stream of keys, in a per-warp buffer of kTopCap keys.
// DISTINCT keeps the 64 least distinct keys.  ENTITY keys hold (rank << 32 | first row of
// the entity) and keep, per entity, its least rank, then the 64 least (rank, first row).

enum TopMode : int32_t { kDistinct = 0, kEntity = 1 };

struct TopSet {
  Key* buf;
  int32_t n;
  int32_t pushed = 0;  // keys offered so far (n can shrink when the buffer compacts)
};

// Sorts buf[0, n) ascending; entries from n to the sorted width are set to max_key().
XG_COLD void top_sort(const Warp& w, Key* buf, int32_t n) {
#if XG_GPU
  int32_t width = 32;
  #pragma unroll 1
  while (width < n) width <<= 1;
  #pragma unroll 1
  for (int32_t i = n + w.lane; i < width; i += 32) buf[i] = max_key();
  #pragma unroll 1
  for (int32_t i = width + w.lane; i < kTopCap; i += 32) buf[i] = max_key();
  __syncwarp();
  #pragma unroll 1
  for (int32_t k = 2; k <= width; k <<= 1) {
    #pragma unroll 1
    for (int32_t j = k >> 1; j > 0; j >>= 1) {
      #pragma unroll 1
      for (int32_t i = w.lane; i < width; i += 32) {
        const int32_t l = i ^ j;
        if (l > i) {
          const Key x = buf[i], y = buf[l];
          const bool up = (i & k) == 0;
          if (up ? key_less(y, x) : key_less(x, y)) {
            buf[i] = y;
            buf[l] = x;
          }
        }
      }
      __syncwarp();
    }
  }
#else
  (void)w;
  std::sort(buf, buf + n, key_less);
  #pragma unroll 1
  for (int32_t i = n; i < kTopCap; ++i) buf[i] = max_key();
#endif
}

// Sorted buf[0, n) -> its first `limit` entries that are distinct (by full key, or by
// the high 32 bits of a when by_high); returns how many were kept.
XG_COLD int32_t top_unique(const Warp& w, Key* buf, int32_t n, int32_t limit, bool by_high) {
#if XG_GPU
  int32_t out = 0;
  Key carry = max_key();
  #pragma unroll 1
  for (int32_t base = 0; base < n && out < limit; base += 32) {
    const Key k = base + w.lane < n ? buf[base + w.lane] : max_key();
    Key prev;
    prev.a = __shfl_up_sync(0xffffffffu, k.a, 1);
    prev.b = __shfl_up_sync(0xffffffffu, k.b, 1);
    prev.pad = 0;
    const Key last = Key{__shfl_sync(0xffffffffu, k.a, 31), __shfl_sync(0xffffffffu, k.b, 31), 0u};
    if (w.lane == 0) prev = carry;
    const bool first = (base == 0 && w.lane == 0);
    const bool same = by_high ? (!first && (prev.a >> 32) == (k.a >> 32)) : (!first && key_eq(prev, k));
    const bool keep = !is_max(k) && !same;
    const uint32_t m = __ballot_sync(0xffffffffu, keep);
    __syncwarp();
    const int32_t pos = out + __popc(m & ((1u << w.lane) - 1u));
    if (keep && pos < limit) buf[pos] = k;
    out += __popc(m);
    carry = last;
    __syncwarp();
  }
  return out < limit ? out : limit;
#else
  (void)w;
  int32_t out = 0;
  #pragma unroll 1
  for (int32_t i = 0; i < n && out < limit; ++i) {
    const Key k = buf[i];
    if (is_max(k)) break;
    if (out > 0) {
      const Key& prev = buf[out - 1];
      if (by_high ? (prev.a >> 32) == (k.a >> 32) : key_eq(prev, k)) continue;
    }
    buf[out++] = k;
  }
  return out;
#endif
}

// The buffer's keys reduced to what the mode keeps, ascending, at most kMaxSet of them.  On
// the device the warp holds the (at most kTopCap) keys in registers, kTopCap / 32 per lane,
// and extracts the least key kMaxSet times (a lane minimum, then a shuffle reduction),
// dropping after each extraction every key equal to it (DISTINCT) or of the same entity
// (ENTITY: the entity's least rank is the first of its keys to be extracted).  That is the
// same function as sorting, keeping the first of each run and truncating, in ~64 short
// rounds of register work instead of two shared-memory bitonic sorts of the whole buffer
// (whose code, rarely run, also came from memory line by line: ~45 us per compaction).
XG_COLD void top_compact(const Warp& w, TopSet& ts, int32_t mode) {
#if XG_GPU
  constexpr int32_t per = kTopCap / 32;
  Key k[per];
#pragma unroll
  for (int32_t j = 0; j < per; ++j) {
    const int32_t i = 32 * j + w.lane;
    k[j] = i < ts.n ? ts.buf[i] : max_key();
  }
  __syncwarp();
  int32_t out = 0;
  #pragma unroll 1
  for (; out < kMaxSet; ++out) {
    Key m = k[0];
#pragma unroll
    for (int32_t j = 1; j < per; ++j)
      if (key_less(k[j], m)) m = k[j];
#pragma unroll
    for (int32_t d = 16; d > 0; d >>= 1) {
      Key o;
      o.a = __shfl_xor_sync(0xffffffffu, m.a, d);
      o.b = __shfl_xor_sync(0xffffffffu, m.b, d);
      o.pad = __shfl_xor_sync(0xffffffffu, m.pad, d);
      if (key_less(o, m)) m = o;
    }
    if (is_max(m)) break;  // (warp-uniform)
    if (w.lane == 0) ts.buf[out] = m;
#pragma unroll
    for (int32_t j = 0; j < per; ++j) {
      const bool same = mode == kEntity ? !is_max(k[j]) && static_cast<uint32_t>(k[j].a) == static_cast<uint32_t>(m.a)
                                        : key_eq(k[j], m);
      if (same) k[j] = max_key();
    }
  }
  ts.n = out;
  __syncwarp();
#else
  if (mode == kEntity) {
    // (rank, row) -> (row, rank): the least rank of each entity comes first.
    warp_for(w, 0, ts.n, [&](int32_t i) {
      const uint64_t a = ts.buf[i].a;
      ts.buf[i].a = (a << 32) | (a >> 32);
    });
    top_sort(w, ts.buf, ts.n);
    int32_t n = top_unique(w, ts.buf, ts.n, kTopCap, true);
    warp_for(w, 0, n, [&](int32_t i) {
      const uint64_t a = ts.buf[i].a;
      ts.buf[i].a = (a << 32) | (a >> 32);
    });
    top_sort(w, ts.buf, n);
    ts.n = n < kMaxSet ? n : kMaxSet;
  } else {
    top_sort(w, ts.buf, ts.n);
    ts.n = top_unique(w, ts.buf, ts.n, kMaxSet, false);
  }
  warp_sync();
#endif
}

// Offer one key per lane (valid lanes only); all lanes call it together.
XG_HD void top_push(const Warp& w, TopSet& ts, bool valid, const Key& k, int32_t mode) {
#if XG_GPU
  const uint32_t m = __ballot_sync(0xffffffffu, valid);
  if (m == 0) return;
  if (ts.n + 32 > kTopCap) top_compact(w, ts, mode);
  const int32_t pos = ts.n + __popc(m & ((1u << w.lane) - 1u));
  if (valid) ts.buf[pos] = k;
  ts.n += __popc(m);
  ts.pushed += __popc(m);
  __syncwarp();
#else
  if (!valid) return;
  if (ts.n + 1 > kTopCap) top_compact(w, ts, mode);
  ts.buf[ts.n++] = k;
  ts.pushed += 1;
#endif
}

// ---------------------------------------------------------------------------------------
// Index reads.

XG_HD int32_t row_len(const Rows& r, int32_t row) { return r.off[row + 1] - r.off[row]; }

// Token of a row at a depth, or -1 past its end (so a row that ends sorts first): one
// read of the column table for the first `cols` depths.
XG_HD int32_t column(const Rows& r, int32_t row, int32_t depth) {
  if (depth < r.cols) return r.col[static_cast<int64_t>(depth) * r.count + row];
  const int32_t a = r.off[row];
  return depth < r.off[row + 1] - a ? r.tok[a + depth] : -1;
}

// The first i in [lo, hi) where pred(i) holds, for a predicate that is false then true
// along the range (hi when it never holds).  On the GPU the warp probes 32 evenly spaced
// rows per round (a 32-ary search: log32 rounds of one parallel load each instead of
// log2 rounds of dependent loads).  lo and hi must be warp-uniform.
template <class P>
XG_HD int32_t warp_partition(const Warp& w, int32_t lo, int32_t hi, P pred) {
#if XG_GPU
  #pragma unroll 1
  while (hi - lo > 32) {
    const int32_t step = (hi - lo + 31) >> 5;
    const int32_t probe = lo + (w.lane + 1) * step - 1;  // the last row of bucket `lane`
    const uint32_t m = __ballot_sync(0xffffffffu, probe >= hi || pred(probe));
    if (m == 0u) return hi;
    const int32_t k = __ffs(m) - 1;  // the first bucket whose last row satisfies pred
    lo += k * step;
    hi = lo + step < hi ? lo + step : hi;
  }
  const int32_t i = lo + w.lane;
  const uint32_t m = __ballot_sync(0xffffffffu, i >= hi || pred(i));
  return m == 0u ? hi : lo + __ffs(m) - 1;
#else
  (void)w;
  #pragma unroll 1
  while (lo < hi) {
    const int32_t mid = lo + ((hi - lo) >> 1);
    if (pred(mid))
      hi = mid;
    else
      lo = mid + 1;
  }
  return lo;
#endif
}

// First row in [lo, hi) whose column at depth is >= token (upper: > token).
XG_SHARED int32_t bound_row(const Warp& w, const Rows& r, int32_t lo, int32_t hi, int32_t depth, int32_t token,
                        bool upper) {
  return warp_partition(w, lo, hi, [&](int32_t row) {
    const int32_t c = column(r, row, depth);
    return upper ? c > token : c >= token;
  });
}

// The rows of [lo, hi) whose column at depth equals token (the typed label extended by it).
XG_SHARED void narrow(const Warp& w, const Rows& r, int32_t& lo, int32_t& hi, int32_t depth, int32_t token) {
  if (depth == 0 && lo == 0 && hi == r.count) {  // the whole index: one table read
    lo = r.first[token];
    hi = r.first[token + 1];
    return;
  }
#if XG_GPU
  if (hi - lo <= 32) {  // both bounds from one load per lane
    const int32_t row = lo + w.lane;
    const int32_t col = row < hi ? column(r, row, depth) : 0x7fffffff;
    const uint32_t ge = __ballot_sync(0xffffffffu, col >= token);
    const uint32_t gt = __ballot_sync(0xffffffffu, col > token);
    const int32_t a = ge ? lo + __ffs(ge) - 1 : hi;
    hi = gt ? lo + __ffs(gt) - 1 : hi;
    lo = a;
    return;
  }
#endif
  const int32_t a = bound_row(w, r, lo, hi, depth, token, false);
  hi = bound_row(w, r, a, hi, depth, token, true);
  lo = a;
}

template <class T>
XG_HD int32_t lower_index(const T* a, int32_t lo, int32_t hi, T value) {
  #pragma unroll 1
  while (lo < hi) {
    const int32_t mid = lo + ((hi - lo) >> 1);
    if (a[mid] < value)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

template <class T>
XG_HD int32_t upper_index(const T* a, int32_t lo, int32_t hi, T value) {
  #pragma unroll 1
  while (lo < hi) {
    const int32_t mid = lo + ((hi - lo) >> 1);
    if (a[mid] <= value)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

XG_HD void prefetch_l1(const void* p) {
#if XG_GPU
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
#else
  (void)p;
#endif
}

struct Edges {
  const int32_t* rel;
  const int32_t* obj;
  const int32_t* first;  // base KG: the edges' folded first rows (edge_first); null for a version's list
  int32_t n;
  int32_t start;         // base KG: index of the first edge
  int32_t run0, runs;    // base KG: the entity's relation runs [run0, run0 + runs); runs -1 otherwise
};

// An entity's adjacency in a KG version: the version's own list for an edited subject,
// else the base CSR slice (src/xgraph/kgversions.py:14-21, the layout both share).
XG_COLD Edges edges_of(const Tables& t, int32_t version, int32_t e) {
  if (version > 0) {
    const int32_t a = t.ver_range[2 * version - 2], b = t.ver_range[2 * version - 1];
    const int32_t at = lower_index(t.ver_subj, a, b, e);
    if (at < b && t.ver_subj[at] == e) {
      const int32_t s = t.ver_adj[at], f = t.ver_adj[at + 1];
      return Edges{t.ver_edge_rel + s, t.ver_edge_obj + s, nullptr, f - s, s, 0, -1};
    }
  }
  const int32_t s = t.adj_off[e], f = t.adj_off[e + 1];
  const int32_t r0 = t.run_off[e], r1 = t.run_off[e + 1];
  return Edges{t.edge_rel + s, t.edge_obj + s, t.edge_first + s, f - s, s, r0, r1 - r0};
}

// First label row of the object of edge i of g (bit 31 of the folded table cleared).
XG_HD int32_t edge_first_row(const Tables& t, const Edges& g, int32_t i) {
  return g.first ? g.first[i] & 0x7fffffff : t.row_first[g.obj[i]];
}

// The objects of one relation within an adjacency list: [first, last) indexes (equal when
// the relation is absent).  In the base KG the entity's relation runs are searched: while
// more than 16 remain, 15 evenly spaced pivots (loaded together) narrow them to one
// bucket; the <= 16 runs left are scanned four (relation, first edge) pairs per round of
// independent loads, so a lookup costs one or two memory round trips with short, rolled
// code.  A version's own list is searched by halving.
XG_COLD void relation_slice(const Tables& t, const Edges& g, int32_t relation, int32_t& first, int32_t& last) {
  first = last = 0;
  if (g.runs < 0) {
    first = lower_index(g.rel, 0, g.n, relation);
    last = upper_index(g.rel, first, g.n, relation);
    return;
  }
  int32_t lo = g.run0, n = g.runs;
#pragma unroll 1
  while (n > 16) {
    const int32_t step = (n + 15) >> 4;
    int32_t skip = 0;
#pragma unroll
    for (int32_t j = 0; j < 15; ++j) {
      const int32_t p = (j + 1) * step;  // bucket j ends before p
      skip += p <= n && t.run_rel[lo + p - 1] < relation;
    }
    lo += skip * step;
    n = n - skip * step < step ? n - skip * step : step;
  }
  // runs[2 k] is run k's relation, runs[2 k + 1] its first edge; the run after the last
  // one of the window closes it (the table ends with a sentinel run)
#pragma unroll 1
  for (int32_t j = 0; j < n; j += 4) {
    int32_t rel[4], at[5];
#pragma unroll
    for (int32_t b = 0; b < 4; ++b) {
      const bool in = j + b < n;
      rel[b] = in ? t.runs[2 * (lo + j + b)] : 0x7fffffff;
      at[b] = in ? t.runs[2 * (lo + j + b) + 1] : 0;
    }
    at[4] = t.runs[2 * (lo + (j + 4 < n ? j + 4 : n)) + 1];
#pragma unroll
    for (int32_t b = 0; b < 4; ++b) {
      if (rel[b] >= relation) {
        if (rel[b] == relation) {
          first = at[b] - g.start;
          last = (b < 3 && j + b + 1 < n ? at[b + 1] : at[4]) - g.start;  // the next run's first edge
        }
        return;
      }
    }
  }
}

XG_HD int32_t degree(const Tables& t, int32_t version, int32_t e) { return edges_of(t, version, e).n; }

// Degree of a label row's owner in the slot's KG version: the row-indexed base table when
// the slot reads the base KG, else the version's list for edited subjects.
XG_HD int32_t row_degree(const Tables& t, int32_t version, int32_t row) {
  return version == 0 ? t.row_degree[row] : degree(t, version, t.ent.owner[row]);
}

// Best-connected order key (src/xgraph/oracle.py:1736-1747): most sitelinks (with the
// sitelink rank), then most adjacency entries in the slot's version, then first row.
// In the base KG both counts come from row-indexed tables (one round of loads, no owner
// hop).
XG_SHARED Key connected_key(const Tables& t, int32_t version, int32_t row) {
  uint32_t links, deg;
  if (version == 0) {
    links = t.row_sitelinks ? static_cast<uint32_t>(t.row_sitelinks[row]) : 0u;
    deg = static_cast<uint32_t>(t.row_degree[row]);
  } else {
    const int32_t e = t.ent.owner[row];
    links = t.sitelinks ? static_cast<uint32_t>(t.sitelinks[e]) : 0u;
    deg = static_cast<uint32_t>(degree(t, version, e));
  }
  return Key{(static_cast<uint64_t>(~links) << 32) | static_cast<uint64_t>(~deg), static_cast<uint32_t>(row), 0u};
}

// ---------------------------------------------------------------------------------------
// One slot's context.

struct Ctx {
  const Tables& t;
  Warp w;
  int32_t slot;
  int32_t* mem;     // slot memory
  Key* top;         // per-warp buffer of kTopCap keys
  int32_t* scratch; // per-warp: kScratchInts ints (slice starts, slice pointers, entity rows)
  // optional copy of the tokens that start the closer, separator and escape (their lists at
  // byte position 0, in that order), e.g. in shared memory; null: read the tables
  const int32_t* delim0 = nullptr;
};

XG_HD int32_t version_of(const Ctx& c) { return c.mem[kMemVersion]; }
XG_HD int32_t reached_count(const Ctx& c) { return c.mem[kMemReached]; }

XG_HD void mem_store(const Ctx& c, int32_t at, int32_t value) {
  if (c.w.leader()) c.mem[at] = value;
}

XG_HD bool has_relation(const Ctx& c, int32_t relation) {
  return (static_cast<uint32_t>(c.mem[kMemHave + (relation >> 5)]) >> (relation & 31)) & 1u;
}

XG_HD bool unbound(const Tables& t, const Ctx& c, const XgState& s) {
  return s.segment == kSubject && (!t.derivation || reached_count(c) == 0);
}

XG_HD bool kept_row(const Tables& t, int32_t row) {
  return !t.kept_prefix || t.kept_prefix[row + 1] > t.kept_prefix[row];
}

// The last closed span was a path (or a plan or comparison): the next span is its answer.
XG_HD bool answers_path(const Tables& t, const XgState& s) {
  return t.paths && (s.last_kind == kPathSpan || s.last_kind == kRelationPlan || s.last_kind == kComparison);
}

// Expressions: the span writes a comparison's operand A (its separator is the operand
// separator).
XG_HD bool operand_a(const XgState& s) { return s.op != 0 && s.segment == kSubject && s.operand == 0; }

// Whether some candidate row of the state's segment lies in [lo, hi)
// (src/xgraph/oracle.py:830-894: _candidates / _segment_candidates).
XG_SHARED bool has_candidate(const Ctx& c, const XgState& s, int32_t lo, int32_t hi) {
  const Tables& t = c.t;
  if (lo >= hi) return false;
  if (s.segment == kSubject) {
    if (unbound(t, c, s)) return !t.kept_prefix || t.kept_prefix[hi] > t.kept_prefix[lo];
    const int32_t* reached = c.mem + kMemReachedRows;
    return warp_any(c.w, 0, reached_count(c), [&](int32_t i) { return reached[i] >= lo && reached[i] < hi; });
  }
  if (s.segment == kRelation) {
    return warp_any(c.w, lo, hi, [&](int32_t row) { return has_relation(c, t.rel.owner[row]); });
  }
  // object: some object row of a (subject, relation) pair in [lo, hi)
  const int32_t subjects = s.subj_hi - s.subj_lo, relations = s.rel_hi - s.rel_lo;
  const int32_t version = version_of(c);
  return warp_any(c.w, 0, subjects * relations, [&](int32_t p) {
    const int32_t e = t.ent.owner[s.subj_lo + p / relations];
    const int32_t r = t.rel.owner[s.rel_lo + p % relations];
    const Edges g = edges_of(t, version, e);
    int32_t a, b;
    relation_slice(t, g, r, a, b);
    const int32_t x = lower_index(g.obj, a, b, lo);
    return x < b && g.obj[x] < hi;
  });
}

// Calls item(valid, owner_index, value) for every element of `count` int32 slices,
// spread over the lanes; slice(k, ptr, len) describes slice k (k < 64).
template <class S, class I>
XG_HD void for_each_slice_item(const Ctx& c, int32_t count, S slice, I item) {
#if XG_GPU
  int32_t* starts = c.scratch;                       // [65]
  const int32_t** ptrs = reinterpret_cast<const int32_t**>(c.scratch + 2 * kMaxSet + 2);  // [64]
  #pragma unroll 1
  for (int32_t base = 0; base < count; base += 64) {
    // slices base + lane and base + 32 + lane, in a loop so that the slice code (often
    // long: an adjacency lookup) appears once
    const int32_t* p0 = nullptr;
    const int32_t* p1 = nullptr;
    int32_t n0 = 0, n1 = 0;
#pragma unroll 1
    for (int32_t h = 0; h < 2; ++h) {
      const int32_t k = base + 32 * h + c.w.lane;
      const int32_t* p = nullptr;
      int32_t n = 0;
      if (k < count) slice(k, p, n);
      if (h == 0) {
        p0 = p;
        n0 = n;
      } else {
        p1 = p;
        n1 = n;
      }
    }
    // inclusive scan of n0 over lanes, then of n1 continuing after the first half
    int32_t x0 = n0, x1 = n1;
    #pragma unroll 1
    for (int32_t d = 1; d < 32; d <<= 1) {
      const int32_t y0 = __shfl_up_sync(0xffffffffu, x0, d);
      const int32_t y1 = __shfl_up_sync(0xffffffffu, x1, d);
      if (c.w.lane >= d) {
        x0 += y0;
        x1 += y1;
      }
    }
    const int32_t half = __shfl_sync(0xffffffffu, x0, 31);
    const int32_t total = half + __shfl_sync(0xffffffffu, x1, 31);
    starts[c.w.lane] = x0 - n0;
    starts[32 + c.w.lane] = half + x1 - n1;
    ptrs[c.w.lane] = p0;
    ptrs[32 + c.w.lane] = p1;
    if (c.w.lane == 0) starts[64] = total;
    __syncwarp();
    // kItemBatch rounds of loads are issued before their items run (item may store, and
    // the compiler would not move a later round's load above that store).
    #pragma unroll 1
    for (int32_t g0 = 0; g0 < total; g0 += 32 * kItemBatch) {
      int32_t k[kItemBatch], value[kItemBatch];
#pragma unroll
      for (int32_t b = 0; b < kItemBatch; ++b) {
        const int32_t g = g0 + 32 * b + c.w.lane;
        k[b] = 0;
        value[b] = 0;
        if (g < total) {
          k[b] = upper_index(starts, 0, 64, g) - 1;
          value[b] = ptrs[k[b]][g - starts[k[b]]];
        }
      }
#pragma unroll
      for (int32_t b = 0; b < kItemBatch; ++b) {
        if (g0 + 32 * b >= total) break;  // warp-uniform
        item(g0 + 32 * b + c.w.lane < total, base + k[b], value[b]);
      }
    }
    __syncwarp();
  }
#else
  #pragma unroll 1
  for (int32_t k = 0; k < count; ++k) {
    const int32_t* p = nullptr;
    int32_t n = 0;
    slice(k, p, n);
    #pragma unroll 1
    for (int32_t i = 0; i < n; ++i) item(true, k, p[i]);
  }
#endif
}

// Writes the bitmap of relations that the entities entity[0, n) have.  All (entity,
// relation run) pairs are spread over the lanes (edges for a version's own list).
XG_COLD void set_have(const Ctx& c, int32_t n, const int32_t* entity, int32_t* have = nullptr) {
  const Tables& t = c.t;
  if (have == nullptr) have = c.mem + kMemHave;
  warp_for(c.w, 0, t.relation_words, [&](int32_t i) { have[i] = 0; });
  const int32_t version = version_of(c);
  for_each_slice_item(
      c, n,
      [&](int32_t k, const int32_t*& p, int32_t& len) {
        const Edges g = edges_of(t, version, entity[k]);
        if (g.runs >= 0) {  // one bit per relation run
          p = t.run_rel + g.run0;
          len = g.runs;
        } else {
          p = g.rel;
          len = g.n;
        }
      },
      [&](bool valid, int32_t, int32_t relation) {
        if (valid) set_bit(reinterpret_cast<uint32_t*>(have), relation);
      });
  warp_sync();
}

// Next path frontier (src/xgraph/oracle.py:1771-1786): objects of the current frontier
// under every relation of the exact relation-label rows [rlo, rhi), each with the least
// start rank it is reached from, kept to 64 by (rank, first row) or, with union paths,
// by first row.  Leaves the result in c.top[0, n) as ENTITY keys and returns n.  When at
// most 64 edges were found no cap applies and no sort is needed: the keys stay as found,
// an entity possibly more than once (once per rank it is reached with).  Every reader
// treats the list as a set with least ranks, so the duplicates change nothing.
// (ents, ranks, count: another frontier than the slot's path frontier, a comparison's
// operand B.)
XG_COLD int32_t next_frontier(const Ctx& c, int32_t rlo, int32_t rhi, const int32_t* ents = nullptr,
                              const int32_t* ranks = nullptr, int32_t count = 0) {
  const Tables& t = c.t;
  const int32_t version = version_of(c);
  if (ents == nullptr) {
    ents = c.mem + kMemFrontierEnt;
    ranks = c.mem + kMemFrontierRank;
    count = c.mem[kMemFrontier];
  }
  const bool folded = version == 0;  // every list is a base-KG slice with folded first rows
  TopSet ts{c.top, 0};
  #pragma unroll 1
  for (int32_t rr = rlo; rr < rhi; ++rr) {
    const int32_t relation = t.rel.owner[rr];
    for_each_slice_item(
        c, count,
        [&](int32_t k, const int32_t*& p, int32_t& n) {
          const Edges g = edges_of(t, version, ents[k]);
          int32_t a, b;
          relation_slice(t, g, relation, a, b);
          p = (folded ? g.first : g.obj) + a;
          n = b - a;
        },
        [&](bool valid, int32_t k, int32_t value) {
          Key key{0, 0, 0};
          if (valid) {
            // folded: value is the first row with the no-triples bit; pad 1 = has triples,
            // 2 = has none, 0 = not known here (a version's list)
            const uint32_t first = folded ? static_cast<uint32_t>(value) & 0x7fffffffu
                                          : static_cast<uint32_t>(t.row_first[value]);
            const uint64_t rank = t.committed ? static_cast<uint32_t>(ranks[k]) : 0u;
            key.a = (rank << 32) | first;
            key.pad = folded ? 1u + (static_cast<uint32_t>(value) >> 31) : 0u;
          }
          top_push(c.w, ts, valid, key, kEntity);
        });
  }
  if (ts.pushed > kMaxSet) top_compact(c.w, ts, kEntity);
  return ts.n;
}

// Keep, in c.top[0, n), the keys of the least rank present (committed paths resolve to
// what the best start reaches, src/xgraph/oracle.py:1160-1162); returns how many.
XG_COLD int32_t keep_least_rank(const Ctx& c, int32_t n) {
  const Key least = warp_min(c.w, 0, n, [&](int32_t i) { return Key{c.top[i].a >> 32, 0u, 0u}; });
#if XG_GPU
  int32_t out = 0;
  #pragma unroll 1
  for (int32_t base = 0; base < n; base += 32) {
    const int32_t i = base + c.w.lane;
    const Key k = i < n ? c.top[i] : max_key();
    const bool keep = i < n && (k.a >> 32) == least.a;
    const uint32_t m = __ballot_sync(0xffffffffu, keep);
    __syncwarp();
    if (keep) c.top[out + __popc(m & ((1u << c.w.lane) - 1u))] = k;
    out += __popc(m);
    __syncwarp();
  }
  return out;
#else
  int32_t out = 0;
  #pragma unroll 1
  for (int32_t i = 0; i < n; ++i)
    if ((c.top[i].a >> 32) == least.a) c.top[out++] = c.top[i];
  return out;
#endif
}

#if XG_GPU
// The distinct values among buf[0, n).a (n <= 64, each below 2^31) in ascending order into
// out[0, m); returns m.  A bitonic network over 64 values held two per lane and exchanged
// by shuffles: no shared-memory traffic and ~300 instructions, against a shared-memory
// sort of 16-byte keys.
XG_COLD int32_t sort_unique64(const Warp& w, const Key* buf, int32_t n, int32_t* out) {
  const int32_t lane = w.lane;
  int32_t v0 = lane < n ? static_cast<int32_t>(buf[lane].a) : 0x7fffffff;
  int32_t v1 = lane + 32 < n ? static_cast<int32_t>(buf[lane + 32].a) : 0x7fffffff;
#pragma unroll 1
  for (int32_t k = 2; k <= 64; k <<= 1) {
#pragma unroll 1
    for (int32_t j = k >> 1; j > 0; j >>= 1) {
      if (j == 32) {  // partners in the two halves of the same lane (k == 64: ascending)
        const int32_t lo = v0 < v1 ? v0 : v1;
        v1 = v0 < v1 ? v1 : v0;
        v0 = lo;
        continue;
      }
      const int32_t o0 = __shfl_xor_sync(0xffffffffu, v0, j);
      const int32_t o1 = __shfl_xor_sync(0xffffffffu, v1, j);
      const bool low = (lane & j) == 0;  // this element is the lower index of its pair
      const bool up0 = (lane & k) == 0, up1 = ((lane + 32) & k) == 0;
      v0 = (low == up0) ? (v0 < o0 ? v0 : o0) : (v0 < o0 ? o0 : v0);
      v1 = (low == up1) ? (v1 < o1 ? v1 : o1) : (v1 < o1 ? o1 : v1);
    }
  }
  // keep the first of each run of equal values (index order: lanes of v0, then of v1)
  int32_t p0 = __shfl_up_sync(0xffffffffu, v0, 1);
  int32_t p1 = __shfl_up_sync(0xffffffffu, v1, 1);
  const int32_t last0 = __shfl_sync(0xffffffffu, v0, 31);
  if (lane == 0) p1 = last0;
  const bool keep0 = v0 != 0x7fffffff && (lane == 0 || v0 != p0);
  const bool keep1 = v1 != 0x7fffffff && v1 != p1;
  const uint32_t m0 = __ballot_sync(0xffffffffu, keep0), m1 = __ballot_sync(0xffffffffu, keep1);
  const uint32_t below = (1u << lane) - 1u;
  if (keep0) out[__popc(m0 & below)] = v0;
  if (keep1) out[__popc(m0) + __popc(m1 & below)] = v1;
  __syncwarp();
  return __popc(m0) + __popc(m1);
}
#endif

// The rows of the entities whose first rows are given by keys c.top[0, n) (low 32 bits of
// a), sorted, first 64 (src/xgraph/oracle.py:697-703 _rows_for, capped as reached).
// Writes them to the slot's reached list.
XG_COLD void reach_rows_of_top(const Ctx& c, int32_t n) {
  const Tables& t = c.t;
  int32_t* firsts = c.scratch + 2 * kMaxSet + 2 + 2 * kMaxSet;  // after starts/ptrs
  warp_for(c.w, 0, n, [&](int32_t i) { firsts[i] = static_cast<int32_t>(c.top[i].a & 0xffffffffu); });
  TopSet ts{c.top, 0};
  for_each_slice_item(
      c, n,
      [&](int32_t k, const int32_t*& p, int32_t& len) {
        const int32_t e = t.ent.owner[firsts[k]];
        p = t.ent_rows + t.ent_rows_off[e];
        len = t.ent_rows_off[e + 1] - t.ent_rows_off[e];
      },
      [&](bool valid, int32_t, int32_t row) {
        top_push(c.w, ts, valid, Key{static_cast<uint64_t>(static_cast<uint32_t>(row)), 0u, 0u}, kDistinct);
      });
  int32_t* reached = c.mem + kMemReachedRows;
#if XG_GPU
  if (ts.pushed <= 64) {  // every row is still in the buffer: sort them in registers
    const int32_t m = sort_unique64(c.w, ts.buf, ts.n, reached);
    mem_store(c, kMemReached, m);
    warp_sync();
    return;
  }
#endif
  if (ts.pushed > 1) top_compact(c.w, ts, kDistinct);  // one key or none: nothing to order
  warp_for(c.w, 0, ts.n, [&](int32_t i) { reached[i] = static_cast<int32_t>(ts.buf[i].a); });
  mem_store(c, kMemReached, ts.n);
  warp_sync();
}

// Forget the next frontier cached by frontier_goes_on (the frontier or version changed).
XG_HD void drop_cached_frontier(const Ctx& c) { mem_store(c, kMemPendingLo, -1); }

// Write the frontier held as ENTITY keys in c.top[0, n) into slot memory.
XG_COLD void store_frontier(const Ctx& c, int32_t n) {
  const Tables& t = c.t;
  int32_t* ents = c.mem + kMemFrontierEnt;
  int32_t* ranks = c.mem + kMemFrontierRank;
  warp_for(c.w, 0, n, [&](int32_t i) {
    const uint64_t a = c.top[i].a;
    ents[i] = t.ent.owner[static_cast<int32_t>(a & 0xffffffffu)];
    ranks[i] = static_cast<int32_t>(a >> 32);
  });
  mem_store(c, kMemFrontier, n);
  drop_cached_frontier(c);
  warp_sync();
}

// Candidate rows of the exact label rows [lo, hi) in the subject segment.
XG_HD bool subject_candidate(const Ctx& c, bool bound, int32_t row) {
  if (!bound) return kept_row(c.t, row);
  const int32_t* reached = c.mem + kMemReachedRows;
  const int32_t n = reached_count(c);
  const int32_t at = lower_index(reached, 0, n, row);
  return at < n && reached[at] == row;
}

// The next frontier through relation-label rows [rlo, rhi) into c.top[0, n): the copy
// cached in slot memory when the same label was just tested for the separator flag (the
// frontier has not changed since: every frontier or version change drops the cache),
// else computed.
XG_COLD int32_t cached_frontier(const Ctx& c, int32_t rlo, int32_t rhi) {
  if (c.mem[kMemPendingLo] == rlo && c.mem[kMemPendingHi] == rhi) {
    const int32_t n = c.mem[kMemPendingCount];
    const int32_t* ranks = c.mem + kMemPendingRank;
    const int32_t* firsts = c.mem + kMemPendingFirst;
    warp_for(c.w, 0, n, [&](int32_t i) {
      c.top[i] = Key{(static_cast<uint64_t>(static_cast<uint32_t>(ranks[i])) << 32) | static_cast<uint32_t>(firsts[i]), 0u, 0u};
    });
    return n;
  }
  return next_frontier(c, rlo, rhi);
}

// Whether some entity of the frontier in c.top[0, n) has triples.
XG_COLD bool top_goes_on(const Ctx& c, int32_t n) {
  const Tables& t = c.t;
  const int32_t version = version_of(c);
  return warp_any(c.w, 0, n, [&](int32_t i) {
    const uint32_t known = c.top[i].pad;
    if (known) return known == 1u;
    return row_degree(t, version, static_cast<int32_t>(c.top[i].a & 0xffffffffu)) > 0;
  });
}

// Whether the flags' "separator after a relation" holds in path mode: some entity of the
// capped next frontier has triples.  The frontier is kept for the transition that follows.
XG_COLD bool frontier_goes_on(const Ctx& c, int32_t rlo, int32_t rhi) {
  const int32_t n = next_frontier(c, rlo, rhi);
  const int32_t version = version_of(c);
  const Tables& t = c.t;
  int32_t* ranks = c.mem + kMemPendingRank;
  int32_t* firsts = c.mem + kMemPendingFirst;
  warp_for(c.w, 0, n, [&](int32_t i) {
    ranks[i] = static_cast<int32_t>(c.top[i].a >> 32);
    firsts[i] = static_cast<int32_t>(c.top[i].a & 0xffffffffu);
  });
  if (c.w.leader()) {
    c.mem[kMemPendingLo] = rlo;
    c.mem[kMemPendingHi] = rhi;
    c.mem[kMemPendingCount] = n;
  }
  warp_sync();
  return warp_any(c.w, 0, n, [&](int32_t i) {
    const uint32_t known = c.top[i].pad;
    if (known) return known == 1u;
    return row_degree(t, version, static_cast<int32_t>(c.top[i].a & 0xffffffffu)) > 0;
  });
}

// ---------------------------------------------------------------------------------------
// Expressions: date and value comparisons (src/xgraph/oracle.py:104-133, 1680-1737;
// csrc/engine.cu:547-611, 988-1125 of the reference).

// The date table's index of an entity, or -1 for an entity that is no date.
XG_HD int32_t date_index(const Tables& t, int32_t entity) {
  const int32_t at = lower_index(t.date_entities, 0, t.date_count, entity);
  return at < t.date_count && t.date_entities[at] == entity ? at : -1;
}

XG_HD int32_t delim_step(const Delim& d, int32_t pos, int32_t token);

XG_HD uint32_t ordered(int32_t x) { return static_cast<uint32_t>(x) ^ 0x80000000u; }  // signed order as unsigned
XG_HD int32_t unordered(uint32_t x) { return static_cast<int32_t>(x ^ 0x80000000u); }

// The operator branch after `token` from byte position `pos` (bytes so far those of
// operator `kind`): the new position, with `kind` the first operator the bytes still fit,
// or -1 (src/xgraph/oracle.py:1097-1101; csrc/engine.cu:604-617).
XG_HD int32_t operator_step(const Tables& t, int32_t pos, int32_t& kind, int32_t token) {
  const int32_t from = kind;
  #pragma unroll 1
  for (int32_t j = 0; j < t.operator_count; ++j) {
    if (pos > 0 && t.operator_lcp[from * kMaxOperators + j] < pos) continue;
    const int32_t next = delim_step(t.operators[j], pos, token);
    if (next >= 0) {
      kind = j;
      return next;
    }
  }
  return -1;
}

// An operator may start here: the first token of an unbound span's subject, no operator yet
// (src/xgraph/oracle.py:1669-1678).
XG_HD bool may_operate(const Ctx& c, const XgState& s) {
  return c.t.operator_count > 0 && s.segment == kSubject && s.op == 0 && s.lo >= 0 && s.depth == 0 &&
         reached_count(c) == 0;
}

// The next frontier of a comparison's operand k through relation-label rows [rlo, rhi)
// into c.top (operand A's from the separator test's cache when it holds it).
XG_COLD int32_t operand_next(const Ctx& c, int32_t k, int32_t rlo, int32_t rhi) {
  if (k == 0) return cached_frontier(c, rlo, rhi);
  const int32_t* op = c.mem + c.t.mem_operand;
  return next_frontier(c, rlo, rhi, op + kOpFrontEnt, op + kOpFrontRank, op[kOpFrontCount]);
}

// The least (start rank, first day, last day) over the dated entities of the frontier in
// c.top[0, n) (Key.a: rank and first day, b: last day, both in signed order); max_key()
// when none is a date.
XG_COLD Key dated_pick(const Ctx& c, int32_t n) {
  const Tables& t = c.t;
  return warp_min(c.w, 0, n, [&](int32_t i) {
    const int32_t at = date_index(t, t.ent.owner[static_cast<int32_t>(c.top[i].a & 0xffffffffu)]);
    if (at < 0) return max_key();
    return Key{((c.top[i].a >> 32) << 32) | ordered(t.date_lo[at]), ordered(t.date_hi[at]), 0u};
  });
}

// A value comparison's operand values: the entities of the least rank in the frontier in
// c.top[0, n) (n > 0), each a label row (first row) or, for a date, its date key, into
// values / dated; returns how many, with `rank` the least rank.
XG_COLD int32_t best_values(const Ctx& c, int32_t n, int32_t* values, int32_t* dated, int32_t& rank) {
  const Tables& t = c.t;
  const int32_t m = keep_least_rank(c, n);
  rank = static_cast<int32_t>(c.top[0].a >> 32);
  warp_for(c.w, 0, m, [&](int32_t i) {
    const int32_t row = static_cast<int32_t>(c.top[i].a & 0xffffffffu);
    const int32_t at = date_index(t, t.ent.owner[row]);
    values[i] = at >= 0 ? t.date_keys[at] : row;
    dated[i] = at >= 0 ? 1 : 0;
  });
  warp_sync();
  return m;
}

XG_COLD int32_t compare(const Ctx& c, int32_t op, int32_t lo, int32_t hi, int32_t& a, int32_t& b);

// A comparison's relation label: both frontiers must go on for the separator, and it
// closes where it has a result.
XG_COLD void comparison_flags(const Ctx& c, const XgState& s, bool& separates, bool& closes) {
  if (separates) separates = top_goes_on(c, operand_next(c, 1, s.lo, s.ex_hi));
  int32_t a = 0, b = 0;
  closes = compare(c, s.op, s.lo, s.ex_hi, a, b) >= 0;
}

// A comparison closed after the relation-label rows [lo, hi): -1 where it cannot close,
// else its result -- 0 operand A's start, 1 operand B's, 2 both (undetermined), 3 the
// verdict yes, 4 no (the reference engine's codes, csrc/engine.cu:1782-1815) -- with a and
// b the label rows of the starts the operands commit to (src/xgraph/oracle.py:1680-1737).
XG_COLD int32_t compare(const Ctx& c, int32_t op, int32_t lo, int32_t hi, int32_t& a, int32_t& b) {
  const Tables& t = c.t;
  int32_t* mem = c.mem + t.mem_operand;
  if (op == 3) {  // a value comparison: each operand's best start with any value
    int32_t rank_a = 0, rank_b = 0;
    const int32_t na = operand_next(c, 0, lo, hi);
    if (na == 0) return -1;
    const int32_t ma = best_values(c, na, mem + kOpValues, mem + kOpDated, rank_a);
    const int32_t nb = operand_next(c, 1, lo, hi);
    if (nb == 0) return -1;
    int32_t* values_b = c.scratch;
    int32_t* dated_b = c.scratch + kMaxSet;
    const int32_t mb = best_values(c, nb, values_b, dated_b, rank_b);
    const int32_t* values_a = mem + kOpValues;
    const int32_t* dated_a = mem + kOpDated;
    const bool entities_a = warp_any(c.w, 0, ma, [&](int32_t i) { return dated_a[i] == 0; });
    const bool entities_b = warp_any(c.w, 0, mb, [&](int32_t i) { return dated_b[i] == 0; });
    if (entities_a != entities_b) return -1;  // values of two kinds
    a = mem[kOpStartsA + rank_a];
    b = mem[kOpStartsB + rank_b];
    const bool shared = warp_any(c.w, 0, ma * mb, [&](int32_t p) {
      const int32_t i = p / mb, j = p % mb;
      return dated_a[i] == dated_b[j] && values_a[i] == values_b[j];
    });
    return shared ? 3 : 4;
  }
  // a date comparison: each operand's best start that reaches a date, its earliest date
  const Key pa = dated_pick(c, operand_next(c, 0, lo, hi));
  if (is_max(pa)) return -1;
  const Key pb = dated_pick(c, operand_next(c, 1, lo, hi));
  if (is_max(pb)) return -1;
  a = mem[kOpStartsA + static_cast<int32_t>(pa.a >> 32)];
  b = mem[kOpStartsB + static_cast<int32_t>(pb.a >> 32)];
  const int32_t lo_a = unordered(static_cast<uint32_t>(pa.a & 0xffffffffu)), hi_a = unordered(pa.b);
  const int32_t lo_b = unordered(static_cast<uint32_t>(pb.a & 0xffffffffu)), hi_b = unordered(pb.b);
  const bool a_first = hi_a < lo_b, b_first = hi_b < lo_a;
  if (op == 1) return a_first ? 0 : b_first ? 1 : 2;  // earlier
  return a_first ? 1 : b_first ? 0 : 2;               // later
}

// ---------------------------------------------------------------------------------------
// Residual-goal STOP (src/xgraph/oracle.py:1608-1635; csrc/engine.cu:1001-1072 of the
// reference).

XG_HD uint64_t stop_used(const XgState& s) {
  return static_cast<uint32_t>(s.stop_used_lo) | (static_cast<uint64_t>(static_cast<uint32_t>(s.stop_used_hi)) << 32);
}

XG_HD void set_stop_used(XgState& s, uint64_t mask) {
  s.stop_used_lo = static_cast<int32_t>(mask);
  s.stop_used_hi = static_cast<int32_t>(mask >> 32);
}

XG_HD bool stop_installed(const Ctx& c) { return c.t.stop_on != nullptr && c.t.stop_on[c.slot] != 0; }

// The slot's STOP entry of relation number r: (answer-head flag, coverage low, high).
XG_HD const int32_t* stop_entry(const Ctx& c, int32_t r) {
  return c.t.stop_rel + (static_cast<int64_t>(c.slot) * c.t.relations + r) * 3;
}

XG_HD uint64_t stop_coverage(const int32_t* e) {
  return static_cast<uint32_t>(e[1]) | (static_cast<uint64_t>(static_cast<uint32_t>(e[2])) << 32);
}

// The question words the relations of relation-label rows [lo, hi) cover (every relation
// the written label names, as the reference's consumed relations read them).
XG_COLD uint64_t stop_consumed(const Ctx& c, int32_t lo, int32_t hi) {
  uint64_t used = 0;
  warp_for(c.w, lo, hi, [&](int32_t row) { used |= stop_coverage(stop_entry(c, c.t.rel.owner[row])); });
#if XG_GPU
  for (int32_t d = 16; d > 0; d >>= 1) used |= __shfl_xor_sync(0xffffffffu, used, d);
#endif
  return used;
}

// The question words among the words of entity label row `row` (the written start).
XG_COLD uint64_t stop_start_words(const Ctx& c, int32_t row) {
  const Tables& t = c.t;
  const int32_t* offsets = t.stop_woff + static_cast<int64_t>(c.slot) * (kMaxStopWords + 2);
  const uint8_t* words = t.stop_words + static_cast<int64_t>(c.slot) * kMaxStopBytes;
  const int32_t count = offsets[0];
  uint64_t used = 0;
  // the row's words one after another; lanes take the question words
  int64_t at = t.stop_label_off[row];
  const int64_t end = t.stop_label_off[row + 1];
#pragma unroll 1
  while (at < end) {
    int64_t stop = at;
    while (stop < end && t.stop_label_words[stop] != 0) ++stop;
    warp_for(c.w, 0, count, [&](int32_t k) {
      const int32_t first = offsets[k + 1], last = offsets[k + 2];
      if (stop - at != last - first) return;
      int32_t j = 0;
      while (j < last - first && words[first + j] == t.stop_label_words[at + j]) ++j;
      if (j == last - first) used |= uint64_t{1} << k;
    });
    at = stop + 1;
  }
#if XG_GPU
  for (int32_t d = 16; d > 0; d >>= 1) used |= __shfl_xor_sync(0xffffffffu, used, d);
#endif
  return used;
}

// Whether STOP holds after the complete relation label rows [s.lo, s.ex_hi) of a path: one
// of their relations is named by the answer head, and no relation of the new, whole
// capped frontier covers a question word that neither the start nor the relations written
// so far (these included) cover.
XG_COLD bool residual_goal_stop(const Ctx& c, const XgState& s) {
  const Tables& t = c.t;
  if (!t.paths || s.segment != kRelation || !stop_installed(c)) return false;
  if (!warp_any(c.w, s.lo, s.ex_hi, [&](int32_t row) { return stop_entry(c, t.rel.owner[row])[0] != 0; }))
    return false;
  const uint64_t used = stop_used(s) | stop_consumed(c, s.lo, s.ex_hi);
  const int32_t n = cached_frontier(c, s.lo, s.ex_hi);  // ENTITY keys in c.top[0, n)
  const int32_t version = version_of(c);
  bool open = false;  // some frontier relation covers an unused question word
  for_each_slice_item(
      c, n,
      [&](int32_t k, const int32_t*& p, int32_t& len) {
        const Edges g = edges_of(t, version, t.ent.owner[static_cast<int32_t>(c.top[k].a & 0xffffffffu)]);
        if (g.runs >= 0) {  // one entry per relation run
          p = t.run_rel + g.run0;
          len = g.runs;
        } else {
          p = g.rel;
          len = g.n;
        }
      },
      [&](bool valid, int32_t, int32_t relation) {
        if (valid && (stop_coverage(stop_entry(c, relation)) & ~used) != 0) open = true;
      });
#if XG_GPU
  open = __any_sync(0xffffffffu, open);
#endif
  return !open;
}

// ---------------------------------------------------------------------------------------
// Weaker relation supports (src/xgraph/oracle.py:67-79, 865-878, 1060-1078, 1809-1822): a
// relation segment's candidates are the relations in the slot memory's relation bitmap --
// every relation (vocabulary support, and a path's first relation under successor
// support), or the successors of the preceding label's supported relations.

XG_HD const uint32_t* successor_row(const Ctx& c, int32_t relation) {
  const int32_t version = version_of(c);
  const int32_t table = version < c.t.successor_tables ? version : 0;
  return c.t.successors + (static_cast<int64_t>(table) * c.t.relations + relation) * c.t.relation_words;
}

// Whether a separator may follow the exact relation label rows [lo, hi): vocabulary
// support, some relation exists; successor support, some supported relation of the label
// has a successor.
XG_COLD bool relation_goes_on(const Ctx& c, int32_t lo, int32_t hi) {
  const Tables& t = c.t;
  if (t.relation_mode == kVocabularySupport) return t.rel.count > 0;
  const int32_t rw = t.relation_words;
  if (t.successors == nullptr) return false;  // (no tables set: no successor)
  return warp_any(c.w, 0, (hi - lo) * rw, [&](int32_t i) {
    const int32_t relation = t.rel.owner[lo + i / rw];
    return has_relation(c, relation) && successor_row(c, relation)[i % rw] != 0u;
  });
}

// The relation bitmap of the next relation segment: every relation (all), or the union of
// the successors of the supported relations of the label rows [lo, hi), computed from the
// old bitmap (a copy in the warp's scratch) before it is replaced.
XG_COLD void next_support(const Ctx& c, int32_t lo, int32_t hi, bool all) {
  const Tables& t = c.t;
  const int32_t rw = t.relation_words;
  int32_t* have = c.mem + kMemHave;
  int32_t* old = c.scratch;  // rw <= kScratchInts (the host refuses more relations)
  const uint32_t tail = (t.relations & 31) ? (1u << (t.relations & 31)) - 1u : ~0u;
  if (all) {
    warp_for(c.w, 0, rw, [&](int32_t w) { have[w] = static_cast<int32_t>(w + 1 < rw ? ~0u : tail); });
    warp_sync();
    return;
  }
  warp_for(c.w, 0, rw, [&](int32_t w) { old[w] = have[w]; });
  warp_sync();
  warp_for(c.w, 0, rw, [&](int32_t w) {
    uint32_t word = 0u;
    for (int32_t row = lo; row < hi; ++row) {
      const int32_t relation = t.rel.owner[row];
      if (t.successors && ((static_cast<uint32_t>(old[relation >> 5]) >> (relation & 31)) & 1u))
        word |= successor_row(c, relation)[w];
    }
    have[w] = static_cast<int32_t>(word);
  });
  warp_sync();
}

// Which delimiter branches may start after the state's typed label
// (src/xgraph/oracle.py:1039-1113: closes, separates, and the escape condition).
XG_SHARED void set_flags(const Ctx& c, XgState& s) {
  const Tables& t = c.t;
  s.flags = 0;
  if (s.lo < 0) {
    s.ex_hi = -1;
    return;
  }
  const Rows& rows = s.segment == kRelation ? t.rel : t.ent;
  s.ex_hi = s.depth == 0 ? s.lo : bound_row(c.w, rows, s.lo, s.hi, s.depth, 0, false);
  const bool bound = s.segment == kSubject && !unbound(t, c, s);
  if (has_candidate(c, s, s.lo, s.ex_hi)) {
    // a comparison closes only after a relation label, where it has a result (below)
    bool closes = (s.segment != kRelation || t.paths) && s.op == 0;
    if (closes && s.segment == kObject && !t.repeats) {
      const int32_t* facts = c.mem + kMemFactRows;
      const int32_t subj = s.subj_key, rel = s.rel_lo, obj = s.lo;
      closes = !warp_any(c.w, 0, c.mem[kMemFacts], [&](int32_t i) {
        return facts[3 * i] == subj && facts[3 * i + 1] == rel && facts[3 * i + 2] == obj;
      });
    }
    bool separates = false;
    if (s.segment == kSubject) {
      const int32_t version = version_of(c);
      separates = !answers_path(t, s) && warp_any(c.w, s.lo, s.ex_hi, [&](int32_t row) {
                    return subject_candidate(c, bound, row) && row_degree(t, version, row) > 0;
                  });
    } else if (s.segment == kRelation) {
      separates = !t.paths || (s.hops < kMaxHops && (t.relation_mode != kFrontierSupport
                                                         ? relation_goes_on(c, s.lo, s.ex_hi)
                                                         : frontier_goes_on(c, s.lo, s.ex_hi)));
      if (s.op != 0) comparison_flags(c, s, separates, closes);
      // residual-goal STOP (src/xgraph/oracle.py:1081-1111): only the closer or the label
      // goes on (neither the separator nor the escape marker starts or goes on)
      if (closes && s.op == 0 && t.stop_on != nullptr && residual_goal_stop(c, s)) {
        s.flags |= kStop;
        separates = false;
      }
    }
    if (closes) s.flags |= kMayClose;
    if (separates) s.flags |= kMaySep;
  }
  // escape (src/xgraph/oracle.py:1874-1883): a bound subject escapes only with bound_escapes
  if (t.escapes && (t.bound_escapes || !bound) && !(s.flags & kStop)) s.flags |= kMayEsc;
}

XG_HD void clear_span(XgState& s) {
  s.segment = kSubject;
  s.depth = 0;
  s.lo = s.hi = 0;
  s.close_pos = s.close_lo = s.close_hi = 0;
  s.sep_pos = s.sep_lo = s.sep_hi = 0;
  s.esc_pos = 0;
  s.subj_lo = s.subj_hi = s.rel_lo = s.rel_hi = s.subj_key = s.hops = 0;
  s.op_pos = s.op_kind = s.op = s.operand = 0;
  s.ex_hi = 0;
  s.flags = 0;
}

// The state right after the span opener (src/xgraph/oracle.py:706-724).
XG_HD void open_span(const Ctx& c, XgState& s) {
  clear_span(s);
  s.phase = kSpan;
  s.pos = 0;
  s.hi = c.t.ent.count;
  s.stop_used_lo = s.stop_used_hi = 0;
  set_flags(c, s);
}

XG_HD void end_span(XgState& s, int32_t phase) {
  clear_span(s);
  s.phase = phase;
  s.pos = 0;
}

// The separator completed after the label rows [llo, lhi) (src/xgraph/oracle.py:1805-1922).
XG_COLD void next_segment(const Ctx& c, XgState& s, int32_t llo, int32_t lhi) {
  const Tables& t = c.t;
  const int32_t version = version_of(c);
  if (s.segment == kSubject) {
    const bool bound = !unbound(t, c, s);
    if (t.paths && t.relation_mode != kFrontierSupport) {
      // no execution frontier: the start keeps its admission, and the first relation may
      // be any (src/xgraph/oracle.py:1809-1822)
      mem_store(c, kMemFrontier, 0);
      drop_cached_frontier(c);
      warp_sync();
      next_support(c, llo, lhi, true);
      s.subj_lo = llo;
      s.subj_hi = lhi;
    } else if (t.paths) {
      // starts: every candidate with triples in best-connected order, kept to 64
      TopSet ts{c.top, 0};
      #pragma unroll 1
      for (int32_t base = llo; base < lhi; base += 32) {
#if XG_GPU
        const int32_t row = base + c.w.lane;
        const bool valid = row < lhi && subject_candidate(c, bound, row) && row_degree(t, version, row) > 0;
        Key k{0, 0, 0};
        if (valid) {
          if (t.committed)
            k = connected_key(t, version, row);
          else
            k = Key{static_cast<uint64_t>(static_cast<uint32_t>(t.row_first[row])), 0u, 0u};
        }
        top_push(c.w, ts, valid, k, kDistinct);
#else
        #pragma unroll 1
        for (int32_t row = base; row < lhi && row < base + 32; ++row) {
          const bool valid = subject_candidate(c, bound, row) && row_degree(t, version, row) > 0;
          if (!valid) continue;
          const Key k = t.committed ? connected_key(t, version, row)
                                    : Key{static_cast<uint64_t>(static_cast<uint32_t>(t.row_first[row])), 0u, 0u};
          top_push(c.w, ts, true, k, kDistinct);
        }
#endif
      }
      if (ts.pushed > 1) top_compact(c.w, ts, kDistinct);  // one key or none: nothing to order
      // a comparison's operand B ranks its starts into the operand region (operand A's
      // frontier stays the path frontier); each operand keeps its ranked starts
      int32_t* op = c.mem + t.mem_operand;
      const bool second = s.op != 0 && s.operand == 1;
      int32_t* ents = second ? op + kOpFrontEnt : c.mem + kMemFrontierEnt;
      int32_t* ranks = second ? op + kOpFrontRank : c.mem + kMemFrontierRank;
      int32_t* starts = s.op == 0 ? nullptr : op + (second ? kOpStartsB : kOpStartsA);
      const int32_t n = ts.n;
      warp_for(c.w, 0, n, [&](int32_t i) {
        if (t.committed) {
          ents[i] = t.ent.owner[static_cast<int32_t>(c.top[i].b)];
          ranks[i] = i;
        } else {
          ents[i] = t.ent.owner[static_cast<int32_t>(c.top[i].a & 0xffffffffu)];
          ranks[i] = 0;
        }
        if (starts) starts[i] = static_cast<int32_t>(c.top[i].b);  // the written label row
      });
      if (second) {
        mem_store(c, t.mem_operand + kOpFrontCount, n);
      } else {
        mem_store(c, kMemFrontier, n);
        drop_cached_frontier(c);
      }
      warp_sync();
      if (s.op != 0 && s.operand == 0) {  // operand A written: operand B follows
        s.operand = 1;
        s.op_pos = s.op_kind = 0;
        s.depth = 0;
        s.lo = 0;
        s.hi = t.ent.count;
        s.close_pos = s.close_lo = s.close_hi = 0;
        s.sep_pos = s.sep_lo = s.sep_hi = 0;
        s.esc_pos = 0;
        set_flags(c, s);
        return;
      }
      if (second) {  // the relations both frontiers have
        set_have(c, c.mem[kMemFrontier], c.mem + kMemFrontierEnt);
        set_have(c, n, ents, op + kOpHave);
        int32_t* have = c.mem + kMemHave;
        warp_for(c.w, 0, t.relation_words, [&](int32_t w) { have[w] &= op[kOpHave + w]; });
        warp_sync();
      } else {
        set_have(c, n, ents);
      }
      s.subj_lo = llo;
      s.subj_hi = lhi;
    } else if (t.derivation) {
      // one subject: the best-connected candidate with triples
      const Key best = warp_min(c.w, llo, lhi, [&](int32_t row) {
        if (!subject_candidate(c, bound, row) || row_degree(t, version, row) == 0) return max_key();
        return connected_key(t, version, row);
      });
      const int32_t row = static_cast<int32_t>(best.b);
      s.subj_lo = row;
      s.subj_hi = row + 1;
      set_have(c, 1, t.ent.owner + row);
    } else {
      s.subj_lo = llo;
      s.subj_hi = lhi;
      set_have(c, lhi - llo, t.ent.owner + llo);
    }
    s.subj_key = llo;
    s.segment = kRelation;
    s.hops = 1;
    // STOP: the question words the written start covers (csrc/engine.cu:1872)
    if (stop_installed(c) && s.op == 0) set_stop_used(s, stop_start_words(c, llo));
  } else if (t.paths && t.relation_mode != kFrontierSupport) {
    if (t.relation_mode == kSuccessorSupport) next_support(c, llo, lhi, false);
    s.hops += 1;
  } else if (t.paths) {
    // STOP: and those the relations just written cover (csrc/engine.cu:1902-1904)
    if (stop_installed(c)) set_stop_used(s, stop_used(s) | stop_consumed(c, llo, lhi));
    const int32_t n = cached_frontier(c, llo, lhi);
    store_frontier(c, n);
    const int32_t* ents = c.mem + kMemFrontierEnt;
    set_have(c, n, ents);
    if (s.op != 0) {  // a comparison: operand B's frontier goes on in lock step
      int32_t* op = c.mem + t.mem_operand;
      const int32_t nb = operand_next(c, 1, llo, lhi);
      warp_for(c.w, 0, nb, [&](int32_t i) {
        op[kOpFrontEnt + i] = t.ent.owner[static_cast<int32_t>(c.top[i].a & 0xffffffffu)];
        op[kOpFrontRank + i] = static_cast<int32_t>(c.top[i].a >> 32);
      });
      mem_store(c, t.mem_operand + kOpFrontCount, nb);
      warp_sync();
      set_have(c, nb, op + kOpFrontEnt, op + kOpHave);
      int32_t* have = c.mem + kMemHave;
      warp_for(c.w, 0, t.relation_words, [&](int32_t w) { have[w] &= op[kOpHave + w]; });
      warp_sync();
    }
    s.hops += 1;
  } else {
    s.rel_lo = llo;
    s.rel_hi = lhi;
    s.segment = kObject;
  }
  warp_sync();
  s.op_pos = s.op_kind = 0;
  s.depth = 0;
  s.lo = 0;
  s.hi = s.segment == kRelation ? t.rel.count : t.ent.count;
  s.close_pos = s.close_lo = s.close_hi = 0;
  s.sep_pos = s.sep_lo = s.sep_hi = 0;
  s.esc_pos = 0;
  set_flags(c, s);
}

// The closer completed after the label rows [llo, lhi) (src/xgraph/oracle.py:1115-1214).
XG_COLD void close_span(const Ctx& c, XgState& s, int32_t llo, int32_t lhi) {
  const Tables& t = c.t;
  const int32_t version = version_of(c);
  if (s.segment == kRelation && s.op != 0) {  // a comparison ends (src/xgraph/oracle.py:1115-1130)
    int32_t a = -1, b = -1;
    const int32_t result = compare(c, s.op, llo, lhi, a, b);
    // the result binds the answer: the rows of its entities (both starts, undetermined; the
    // verdict's entity, a value comparison)
    const int32_t ea = a >= 0 ? t.ent.owner[a] : -1, eb = b >= 0 ? t.ent.owner[b] : -1;
    const int32_t first = result < 0 ? -1 : result == 1 ? eb : result == 3 ? t.verdict_yes
                                          : result == 4 ? t.verdict_no : ea;
    const int32_t second = result == 2 ? eb : -1;
    int32_t n = 0;
    for (const int32_t e : {first, second}) {  // (an entity without label rows binds nothing)
      const int32_t row = e >= 0 && e < t.entities ? t.ent_first_row[e] : -1;
      if (row < 0) continue;
      if (c.w.leader()) c.top[n] = Key{static_cast<uint32_t>(row), 0u, 0u};
      ++n;
    }
    warp_sync();
    reach_rows_of_top(c, n);
    drop_cached_frontier(c);
    warp_sync();
    s.last_kind = kComparison;
    s.last_lo = a;
    s.last_hi = b;
    s.last_subj_lo = result;
    s.last_subj_hi = s.op;
    s.last_rel_lo = s.last_rel_hi = 0;
  } else if (s.segment == kRelation && t.relation_mode != kFrontierSupport) {
    // a plan under a weaker support: unresolved, nothing executed or bound
    // (src/xgraph/oracle.py:1138-1147)
    if (c.w.leader()) c.mem[kMemReached] = c.mem[kMemFrontier] = 0;
    drop_cached_frontier(c);
    warp_sync();
    s.last_kind = kRelationPlan;
    s.last_lo = s.last_hi = s.last_subj_lo = s.last_subj_hi = s.last_rel_lo = s.last_rel_hi = 0;
  } else if (s.segment == kRelation) {  // a path ends
    int32_t n = cached_frontier(c, llo, lhi);
    if (t.committed && n > 0) n = keep_least_rank(c, n);
    reach_rows_of_top(c, n);
    s.last_kind = kPathSpan;
    s.last_lo = s.last_hi = s.last_subj_lo = s.last_subj_hi = s.last_rel_lo = s.last_rel_hi = 0;
  } else if (s.segment == kSubject) {
    const bool bound = !unbound(t, c, s);
    s.answer_complete = t.end_after_answer && answers_path(t, s) ? 1 : 0;
    if (bound) {  // one entity: the best-connected candidate
      const Key best = warp_min(c.w, llo, lhi, [&](int32_t row) {
        return subject_candidate(c, true, row) ? connected_key(t, version, row) : max_key();
      });
      const int32_t row = static_cast<int32_t>(best.b);
      s.last_lo = row;
      s.last_hi = row + 1;
      s.last_subj_lo = row;
    } else {
      s.last_lo = llo;
      s.last_hi = lhi;
      s.last_subj_lo = -1;
    }
    s.last_kind = kEntitySpan;
    s.last_subj_hi = s.last_rel_lo = s.last_rel_hi = 0;
  } else {  // a fact span
    const int32_t facts = c.mem[kMemFacts];
    if (facts < kMaxSet && c.w.leader()) {
      c.mem[kMemFactRows + 3 * facts] = s.subj_key;
      c.mem[kMemFactRows + 3 * facts + 1] = s.rel_lo;
      c.mem[kMemFactRows + 3 * facts + 2] = llo;
      c.mem[kMemFacts] = facts + 1;
    }
    warp_sync();
    if (t.derivation) {  // reached: every row of the objects with the label (_reached)
      const int32_t relations = s.rel_hi - s.rel_lo;
      TopSet ts{c.top, 0};
      // entities reached, as first rows, kept distinct (at most 64 needed for 64 rows)
      #pragma unroll 1
      for (int32_t p = 0; p < (s.subj_hi - s.subj_lo) * relations; ++p) {
        const int32_t e = t.ent.owner[s.subj_lo + p / relations];
        const int32_t r = t.rel.owner[s.rel_lo + p % relations];
        const Edges g = edges_of(t, version, e);
        int32_t a, b;
        relation_slice(t, g, r, a, b);
        const int32_t x = lower_index(g.obj, a, b, llo);
        const int32_t y = lower_index(g.obj, x, b, lhi);
        #pragma unroll 1
        for (int32_t base = x; base < y; base += 32) {
#if XG_GPU
          const int32_t i = base + c.w.lane;
          const bool valid = i < y;
          Key k{0, 0, 0};
          if (valid) k.a = static_cast<uint32_t>(edge_first_row(t, g, i));
          top_push(c.w, ts, valid, k, kDistinct);
#else
          #pragma unroll 1
          for (int32_t i = base; i < y && i < base + 32; ++i)
            top_push(c.w, ts, true, Key{static_cast<uint32_t>(edge_first_row(t, g, i)), 0u, 0u}, kDistinct);
#endif
        }
      }
      if (ts.pushed > 1) top_compact(c.w, ts, kDistinct);  // one key or none: nothing to order
      reach_rows_of_top(c, ts.n);
    }
    s.last_kind = kFactSpan;
    s.last_lo = llo;
    s.last_hi = lhi;
    s.last_subj_lo = s.subj_lo;
    s.last_subj_hi = s.subj_hi;
    s.last_rel_lo = s.rel_lo;
    s.last_rel_hi = s.rel_hi;
  }
  end_span(s, kFree);
}

// Next byte position of delimiter `which` (0 closer, 1 separator, 2 escape) after
// `token` from byte position `pos`, or -1 when the token does not continue it.
XG_HD int32_t delim_next(const Tables& t, uint64_t packed, int32_t which, int32_t pos, int32_t token);

XG_HD int32_t delim_step(const Delim& d, int32_t pos, int32_t token) {
  const int32_t a = delim_begin(d, pos), b = delim_end(d, pos);
  const int32_t at = lower_index(d.tok, a, b, token);
  return at < b && d.tok[at] == token ? d.next[at] : -1;
}

XG_HD int32_t delim_next(const Tables& t, uint64_t packed, int32_t which, int32_t pos, int32_t token) {
  if (t.dstep) {
    const int32_t offset = which == 0 ? 0 : which == 1 ? t.closer.len : t.closer.len + t.separator.len;
    const int32_t next = static_cast<int32_t>((packed >> (4 * (offset + pos))) & 15u);
    return next ? next : -1;
  }
  return delim_step(which == 0 ? t.closer : which == 1 ? t.separator : t.escape, pos, token);
}

// Expressions, out of the per-token path (most engines have none): the operand
// separator's step, the operator branch after a token (alive, or starting at an unbound
// span's first token; kind: the operator the bytes fit), and the span after a complete
// operator (src/xgraph/oracle.py:1097-1101, 1235-1246).
XG_COLD int32_t operand_sep_step(const Tables& t, int32_t pos, int32_t token) {
  return delim_step(t.operand_sep, pos, token);
}

XG_COLD int32_t operator_branch(const Ctx& c, const XgState& s, int32_t token, int32_t& kind) {
  if (s.op_pos > 0) return operator_step(c.t, s.op_pos, kind, token);
  if (!may_operate(c, s)) return -1;
  kind = 0;
  return operator_step(c.t, 0, kind, token);
}

XG_COLD void start_operand_a(const Ctx& c, XgState& s, int32_t kind) {
  clear_span(s);
  s.pos = 0;
  s.hi = c.t.ent.count;
  s.op = kind + 1;
  s.stop_used_lo = s.stop_used_hi = 0;
  set_flags(c, s);
}

// One token inside a span (src/xgraph/oracle.py:896-1263, in-scope branches).
XG_HD void advance_span(const Ctx& c, XgState& s, int32_t token) {
  const Tables& t = c.t;
  int32_t close = -1, sep = -1, esc = -1, op = -1, op_kind = s.op_kind;
  int32_t close_lo = s.close_lo, close_hi = s.close_hi, sep_lo = s.sep_lo, sep_hi = s.sep_hi;
  const uint64_t packed = t.dstep ? t.dstep[token] : 0u;
  // expressions: operand A of a comparison takes the operand separator in the separator's
  // place
  const bool first_operand = t.operator_count > 0 && operand_a(s);
  const int32_t sep_len = first_operand ? t.operand_sep.len : t.separator.len;
  if (s.close_pos > 0) {
    close = delim_next(t, packed, 0, s.close_pos, token);
  } else if (s.flags & kMayClose) {
    close = delim_next(t, packed, 0, 0, token);
    close_lo = s.lo;
    close_hi = s.ex_hi;
  }
  if (s.sep_pos > 0 && !(s.flags & kStop)) {
    sep = first_operand ? operand_sep_step(t, s.sep_pos, token) : delim_next(t, packed, 1, s.sep_pos, token);
  } else if (s.flags & kMaySep) {
    sep = first_operand ? operand_sep_step(t, 0, token) : delim_next(t, packed, 1, 0, token);
    sep_lo = s.lo;
    sep_hi = s.ex_hi;
  }
  if (t.operator_count > 0) op = operator_branch(c, s, token, op_kind);
  if (s.esc_pos > 0 && !(s.flags & kStop)) {
    esc = delim_next(t, packed, 2, s.esc_pos, token);
  } else if (s.flags & kMayEsc) {
    esc = delim_next(t, packed, 2, 0, token);
  }
  int32_t lo = -1, hi = -1;
  if (s.lo >= 0) {
    const Rows& rows = s.segment == kRelation ? t.rel : t.ent;
    lo = s.lo;
    hi = s.hi;
    narrow(c.w, rows, lo, hi, s.depth, token);
    if (!has_candidate(c, s, lo, hi)) lo = hi = -1;
  }
  if (close == t.closer.len) {
    close_span(c, s, close_lo, close_hi);
    return;
  }
  if (sep == sep_len) {
    next_segment(c, s, sep_lo, sep_hi);
    return;
  }
  if (esc == t.escape.len) {
    end_span(s, kEscaped);
    return;
  }
  if (op >= 0 && op == t.operators[op_kind].len) {
    start_operand_a(c, s, op_kind);
    return;
  }
  if (lo < 0 && close < 0 && sep < 0 && esc < 0 && op < 0) {
    s.phase = kError;
    return;
  }
  s.close_pos = close > 0 ? close : 0;
  s.close_lo = close > 0 ? close_lo : 0;
  s.close_hi = close > 0 ? close_hi : 0;
  s.sep_pos = sep > 0 ? sep : 0;
  s.sep_lo = sep > 0 ? sep_lo : 0;
  s.sep_hi = sep > 0 ? sep_hi : 0;
  s.esc_pos = esc > 0 ? esc : 0;
  s.op_pos = op > 0 ? op : 0;
  s.op_kind = op > 0 ? op_kind : 0;
  if (lo >= 0) {
    s.lo = lo;
    s.hi = hi;
    s.depth += 1;
  } else {
    s.lo = s.hi = -1;
  }
  set_flags(c, s);
}

// Start the loads a label step in this state will need (the current range's columns at the
// typed depth and the next, owners and row degrees, the slot's memory row, the delimiter
// lists) before the token that drives it is known: none depends on the token, and each
// would otherwise be a cold dependent load on the step's critical path.
XG_HD void prefetch_span(const Ctx& c, const XgState& s) {
#if XG_GPU
  const Tables& t = c.t;
  const int32_t lane = c.w.lane;
  const int32_t mem_lines = (t.memory_ints + 31) >> 5;
  if (lane < mem_lines) prefetch_l1(c.mem + lane * 32);
  if (lane < 3) {
    const Delim& d = lane == 0 ? t.closer : lane == 1 ? t.separator : t.escape;
    prefetch_l1(d.tok + d.at[0]);
  }
  if (s.segment == kRelation && t.paths && c.mem[kMemVersion] == 0) {
    // a relation label of a path: the next frontier will read each frontier entity's
    // adjacency and run offsets; start their lines now (the entities' read from the slot's
    // memory overlaps the token's)
    const int32_t count = c.mem[kMemFrontier];
    if (lane < count) {
      const int32_t e = c.mem[kMemFrontierEnt + lane];
      prefetch_l1(t.adj_off + e);
      prefetch_l1(t.run_off + e);
    }
  }
  if (s.lo < 0 || s.hi - s.lo > 64) return;
  const Rows& r = s.segment == kRelation ? t.rel : t.ent;
  #pragma unroll 1
  for (int32_t row = s.lo + lane; row < s.hi; row += 32) {
    if (s.depth < r.cols) prefetch_l1(r.col + static_cast<int64_t>(s.depth) * r.count + row);
    if (s.depth + 1 < r.cols) prefetch_l1(r.col + static_cast<int64_t>(s.depth + 1) * r.count + row);
    prefetch_l1(r.owner + row);
    if (s.segment == kSubject) {
      prefetch_l1(t.row_degree + row);
      if (t.kept_prefix) prefetch_l1(t.kept_prefix + row);
    }
  }
#else
  (void)c;
  (void)s;
#endif
}

XG_HD bool eos_allowed(const Tables& t, int32_t token) {
  return (t.eos_mask[token >> 5] >> (token & 31)) & 1u;
}

// One token of any phase (src/xgraph/oracle.py:759-828).
XG_HD void advance_state(const Ctx& c, XgState& s, int32_t token) {
  const Tables& t = c.t;
  if (s.phase == kError) return;
  if (token < 0 || token >= t.vocab) {
    s.phase = kError;
    return;
  }
  if (s.answer_complete) {
    if (!eos_allowed(t, token)) s.phase = kError;
    return;
  }
  if (s.phase == kFree) {
    const int8_t code = t.free_next[static_cast<int64_t>(s.pos) * t.vocab + token];
    if (code == kReject)
      s.phase = kError;
    else if (code == kComplete)
      open_span(c, s);
    else
      s.pos = code;
  } else if (s.phase == kEscaped) {
    const int8_t code = t.esc_next[static_cast<int64_t>(s.pos) * t.vocab + token];
    if (code == kReject) {
      s.phase = kError;
    } else if (code == kComplete) {
      end_span(s, kFree);
      s.last_kind = kUnresolved;
      s.last_lo = s.last_hi = s.last_subj_lo = s.last_subj_hi = s.last_rel_lo = s.last_rel_hi = 0;
    } else {
      s.pos = code;
    }
  } else {
    advance_span(c, s, token);
  }
}

// ---------------------------------------------------------------------------------------
// Mask of the slot's current state.

XG_HD const uint32_t* wide_mask(const Tables& t, int32_t lo, int32_t depth) {
  if (t.wide_count == 0) return nullptr;
  const int64_t key = static_cast<int64_t>(lo) * 16 + depth;
  const int32_t at = lower_index(t.wide_keys, 0, t.wide_count, key);
  if (at < t.wide_count && t.wide_keys[at] == key) return t.wide_masks + static_cast<int64_t>(at) * t.words_padded;
  return nullptr;
}

// The tokens that continue the closer, separator and escape branches from byte positions
// close, sep and esc (-1: that branch is not live), as one lane-parallel loop over the
// three token lists (their loads issue together).
// (operand: the separator branch matches the operand separator, a comparison's operand A.)
XG_SHARED void add_delimiters(const Ctx& c, int32_t close, int32_t sep, int32_t esc, uint32_t* out,
                              bool operand = false) {
  const Tables& t = c.t;
  const Delim& sd = operand ? t.operand_sep : t.separator;
  const int32_t a0 = close >= 0 ? delim_begin(t.closer, close) : 0;
  const int32_t n0 = close >= 0 ? delim_end(t.closer, close) - a0 : 0;
  const int32_t a1 = sep >= 0 ? delim_begin(sd, sep) : 0;
  const int32_t n1 = sep >= 0 ? delim_end(sd, sep) - a1 : 0;
  const int32_t a2 = esc >= 0 ? delim_begin(t.escape, esc) : 0;
  const int32_t n2 = esc >= 0 ? delim_end(t.escape, esc) - a2 : 0;
  // a branch at its start reads the copied start lists when there is a copy
  const int32_t c0 = t.closer.at[1] - t.closer.at[0], c1 = t.separator.at[1] - t.separator.at[0];
  const int32_t* p0 = c.delim0 && close == 0 ? c.delim0 : t.closer.tok + a0;
  const int32_t* p1 = c.delim0 && sep == 0 && !operand ? c.delim0 + c0 : sd.tok + a1;
  const int32_t* p2 = c.delim0 && esc == 0 ? c.delim0 + c0 + c1 : t.escape.tok + a2;
  warp_for_loaded(
      c.w, 0, n0 + n1 + n2,
      [&](int32_t i) { return i < n0 ? p0[i] : i < n0 + n1 ? p1[i - n0] : p2[i - n0 - n1]; },
      [&](int32_t, int32_t token) { set_bit(out, token); });
}

// Label tokens that keep a live label branch alive: the column at `depth` of every
// candidate row in [lo, hi) that continues past it.
XG_COLD void add_label_tokens(const Ctx& c, const XgState& s, uint32_t* out) {
  const Tables& t = c.t;
  const int32_t d = s.depth, lo = s.lo, hi = s.hi;
  if (s.segment == kSubject) {
    if (unbound(t, c, s)) {
      warp_for_loaded(
          c.w, lo, hi, [&](int32_t row) { return kept_row(t, row) ? column(t.ent, row, d) : -1; },
          [&](int32_t, int32_t tok) {
            if (tok >= 0) set_bit(out, tok);
          });
    } else {
      const int32_t* reached = c.mem + kMemReachedRows;
      warp_for_loaded(
          c.w, 0, reached_count(c),
          [&](int32_t i) {
            const int32_t row = reached[i];
            return row >= lo && row < hi ? column(t.ent, row, d) : -1;
          },
          [&](int32_t, int32_t tok) {
            if (tok >= 0) set_bit(out, tok);
          });
    }
  } else if (s.segment == kRelation) {
    struct TokenOwner {
      int32_t tok, owner;
    };
    warp_for_loaded(
        c.w, lo, hi, [&](int32_t row) { return TokenOwner{column(t.rel, row, d), t.rel.owner[row]}; },
        [&](int32_t, TokenOwner x) {
          if (x.tok >= 0 && has_relation(c, x.owner)) set_bit(out, x.tok);
        });
  } else {
    const int32_t relations = s.rel_hi - s.rel_lo;
    const int32_t version = version_of(c);
    #pragma unroll 1
    for (int32_t p = 0; p < (s.subj_hi - s.subj_lo) * relations; ++p) {
      const int32_t e = t.ent.owner[s.subj_lo + p / relations];
      const int32_t r = t.rel.owner[s.rel_lo + p % relations];
      const Edges g = edges_of(t, version, e);
      int32_t a, b;
      relation_slice(t, g, r, a, b);
      const int32_t x = lower_index(g.obj, a, b, lo);
      const int32_t y = lower_index(g.obj, x, b, hi);
      warp_for(c.w, x, y, [&](int32_t i) {
        const int32_t tok = column(t.ent, g.obj[i], d);
        if (tok >= 0) set_bit(out, tok);
      });
    }
  }
}

// The tokens that continue the operator branch from its byte position (every operator the
// bytes so far fit; at position 0 every operator).
XG_COLD void add_operator_tokens(const Ctx& c, const XgState& s, uint32_t* out) {
  const Tables& t = c.t;
  #pragma unroll 1
  for (int32_t j = 0; j < t.operator_count; ++j) {
    if (s.op_pos > 0 && t.operator_lcp[s.op_kind * kMaxOperators + j] < s.op_pos) continue;
    const Delim& d = t.operators[j];
    warp_for(c.w, delim_begin(d, s.op_pos), delim_end(d, s.op_pos), [&](int32_t i) { set_bit(out, d.tok[i]); });
  }
}

// A mask as base | delta (either may be null; both null: the error phase, nothing masked).
struct MaskRef {
  const uint32_t* base;
  uint32_t* delta;
};

// The mask of a state: outside a span a precomputed table row (base only); inside one the
// root or wide mask of an unbound label range as base (no copy), and the buffer `own`
// (zeroed unless `zeroed`, then the label and delimiter tokens) as delta; in the error
// phase neither.
XG_HD MaskRef compose_mask(const Ctx& c, const XgState& s, uint32_t* own, bool zeroed = false) {
  const Tables& t = c.t;
  const int64_t stride = t.words_padded;
  const uint32_t* base = nullptr;
  uint32_t* delta = nullptr;
  if (s.phase == kFree) {
    base = s.answer_complete ? t.eos_mask : t.free_mask + s.pos * stride;
  } else if (s.phase == kEscaped) {
    base = t.esc_mask + s.pos * stride;
  } else if (s.phase == kSpan) {
    delta = own;
    bool scan = s.lo >= 0;
    if (scan && unbound(t, c, s)) {
      if (s.depth == 0 && s.lo == 0 && s.hi == t.ent.count) {
        base = t.root_mask;
        scan = false;
      } else if ((base = wide_mask(t, s.lo, s.depth)) != nullptr) {
        scan = false;
      }
    }
    if (!zeroed) {  // (a caller may hand over a buffer it has cleared already)
#if XG_GPU
      uint4* to = reinterpret_cast<uint4*>(delta);
      const int32_t quads = t.words_padded >> 2;
#pragma unroll 1
      for (int32_t i = c.w.lane; i < quads; i += 32) to[i] = make_uint4(0u, 0u, 0u, 0u);
      __syncwarp();
#else
#pragma unroll 1
      for (int32_t i = 0; i < t.words_padded; ++i) delta[i] = 0u;
#endif
    }
    if (scan) add_label_tokens(c, s, delta);
    // each delimiter branch: its next tokens from where it stands, or from its start when
    // the flags let it begin here
    const int32_t close = s.close_pos > 0 ? s.close_pos : (s.flags & kMayClose) ? 0 : -1;
    const bool stop = s.flags & kStop;  // STOP: the separator and the escape marker neither go on nor start
    const int32_t sep = s.sep_pos > 0 && !stop ? s.sep_pos : (s.flags & kMaySep) ? 0 : -1;
    const int32_t esc = s.esc_pos > 0 && !stop ? s.esc_pos : (s.flags & kMayEsc) ? 0 : -1;
    add_delimiters(c, close, sep, esc, delta, t.operator_count > 0 && operand_a(s));
    // expressions: the tokens that take the operator branch on (from where it stands, or
    // from its start where an operator may start)
    if (t.operator_count > 0 && (s.op_pos > 0 || may_operate(c, s))) add_operator_tokens(c, s, delta);
    warp_sync();
  }
  return MaskRef{base, delta};
}

// Record the slot's mask for its current state, its own buffer row as the delta.
XG_HD void build_mask(const Ctx& c, const XgState& s) {
  const Tables& t = c.t;
  const MaskRef m = compose_mask(c, s, t.masks + c.slot * static_cast<int64_t>(t.words_padded));
  if (c.w.leader()) {
    t.base[c.slot] = m.base;
    t.delta[c.slot] = m.delta;
  }
}

// ---------------------------------------------------------------------------------------
// apply_mask's logit policies, release and escape bias (csrc/engine.cu:2416-2450 of the
// reference: where a span row's escape marker stands, and which tokens commit to it).

// The byte position the row's escape marker goes on from -- where it stands once started,
// 0 where it may start here (a live label with escapes allowed) -- when some token takes it
// further; -1 outside a span or with no way on.  A released row may write only the
// marker's next tokens from there.
XG_HD int32_t escape_position(const Tables& t, const XgState& s) {
  if (s.phase != kSpan || (s.flags & kStop)) return -1;
  const int32_t pos = s.esc_pos;
  if (delim_end(t.escape, pos) <= delim_begin(t.escape, pos)) return -1;
  return pos > 0 || (s.flags & kMayEsc) ? pos : -1;
}

// f(token), on every lane, for each token that commits the row to the escape marker: where
// the marker may start and has not, each token that starts it and continues neither the
// label nor the separator or closer (live, or startable here).  The tokens are distinct
// and all allowed in the row's mask.
template <class F>
XG_HD void for_each_escape_commit(const Ctx& c, const XgState& s, F f) {
  const Tables& t = c.t;
  if (s.phase != kSpan || s.esc_pos != 0 || !(s.flags & kMayEsc)) return;
  const int32_t close = s.close_pos > 0 ? s.close_pos : (s.flags & kMayClose) ? 0 : -1;
  const int32_t sep = s.sep_pos > 0 ? s.sep_pos : (s.flags & kMaySep) ? 0 : -1;
  const Rows& rows = s.segment == kRelation ? t.rel : t.ent;
  const int32_t a = delim_begin(t.escape, 0), b = delim_end(t.escape, 0);
#pragma unroll 1
  for (int32_t i = a; i < b; ++i) {
    const int32_t token = t.escape.tok[i];
    if (close >= 0 && delim_step(t.closer, close, token) >= 0) continue;
    if (sep >= 0 && delim_step(operand_a(s) ? t.operand_sep : t.separator, sep, token) >= 0) continue;
    int32_t kind = s.op_kind;
    if ((s.op_pos > 0 || may_operate(c, s)) && operator_step(t, s.op_pos, kind, token) >= 0) continue;
    int32_t lo = s.lo, hi = s.hi;
    narrow(c.w, rows, lo, hi, s.depth, token);
    if (has_candidate(c, s, lo, hi)) continue;
    f(token);
  }
}

// ---------------------------------------------------------------------------------------
// Host side of the expression tables (xg_set_expressions, and the host seam's copy).

// One delimiter list of the packed buffer: where its offsets, tokens and next positions
// start in the buffer, its length, and its first offsets (Delim::at).
struct PackedDelim {
  int64_t off, tok, next;
  int32_t len;
  int32_t at[17];
};

// Parses `count` delimiter lists packed one after another in p[0, ints): each its length
// (1..64), its len + 1 CSR offsets (from 0, non-decreasing), then its tokens (in [0,
// vocab), ascending within each byte position) and their next positions (1..len).  False
// when the buffer is malformed or not used up exactly.
inline bool parse_packed_delims(const int32_t* p, int64_t ints, int32_t count, int32_t vocab, PackedDelim* out) {
  int64_t at = 0;
  for (int32_t k = 0; k < count; ++k) {
    if (at >= ints) return false;
    const int32_t len = p[at];
    if (len < 1 || len > 64 || at + 2 + len > ints) return false;
    const int64_t off = at + 1;
    if (p[off] != 0) return false;
    for (int32_t i = 0; i < len; ++i)
      if (p[off + i + 1] < p[off + i]) return false;
    const int64_t n = p[off + len];
    const int64_t tok = off + len + 1, next = tok + n;
    if (next + n > ints) return false;
    for (int32_t i = 0; i < len; ++i) {
      for (int64_t j = p[off + i]; j < p[off + i + 1]; ++j) {
        if (p[tok + j] < 0 || p[tok + j] >= vocab || p[next + j] <= i || p[next + j] > len) return false;
        if (j > p[off + i] && p[tok + j] <= p[tok + j - 1]) return false;
      }
    }
    out[k].off = off;
    out[k].tok = tok;
    out[k].next = next;
    out[k].len = len;
    for (int32_t i = 0; i < 17; ++i) out[k].at[i] = i <= len ? p[off + i] : 0;
    at = next + n;
  }
  return at == ints;
}

// A date key's first (first) or last day, packed with precision bits 0 (xgraph_b200.dates
// date_lo / date_hi).
inline int32_t date_bound(int32_t key, bool first) {
  const int64_t k = key;
  const int64_t year = k >> 11, precision = k & 3;
  int64_t month = (k >> 7) & 15, day = (k >> 2) & 31;
  if (precision == 0 || month == 0) month = first ? 1 : 12;
  if (precision != 2) day = first ? 1 : 31;
  return static_cast<int32_t>(static_cast<uint32_t>(static_cast<uint64_t>((year << 11) | (month << 7) | (day << 2))));
}

}  // namespace xg
