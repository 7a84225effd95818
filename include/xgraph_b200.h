/* xgraph-b200: C ABI of the B200-native KG constraint engine.
 *
 * This is the boundary the reference's Python engine binds through nanobind
 * (csrc/engine.cu:3191-3256, class Engine); here every method is a plain extern "C"
 * function over raw pointers, sizes and a cudaStream_t passed as void*, so any FFI
 * (ctypes, cffi, cgo, JNI) can bind it.  No torch or DLPack type crosses it.
 *
 * Conventions
 *   - Every function returns XG_OK (0) or an error code; xg_last_error() gives the
 *     message of the calling thread's last error.  XG_EINVAL maps to the reference's
 *     std::invalid_argument (Python ValueError), XG_ECUDA to std::runtime_error after
 *     a CUDA failure (the sticky error is cleared, as csrc/engine.cu:210-215 does).
 *   - Device pointers are CUDA device addresses on the engine's device; "host"
 *     arguments are ordinary host memory.  All work is enqueued on `stream`
 *     (NULL = legacy default stream) unless the function says it waits.
 *   - Token masks are uint32 words, bit i of word w = token 32*w + i (little-endian),
 *     as src/xgraph/engine.py:86-94 packs them.
 */
#ifndef XGRAPH_B200_H
#define XGRAPH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XG_ABI_VERSION 4

#if defined(__GNUC__)
#define XG_API __attribute__((visibility("default")))
#else
#define XG_API
#endif

enum xg_status {
  XG_OK = 0,
  XG_EINVAL = 1,  /* invalid argument (reference: std::invalid_argument -> ValueError) */
  XG_ECUDA = 2,   /* a CUDA call failed (reference: std::runtime_error) */
  XG_ENOMEM = 3,  /* a device allocation failed */
};

enum xg_dtype { XG_F32 = 0, XG_BF16 = 1, XG_F16 = 2 };

/* Per-slot constraint state: 64 int32 words.  The first 31 fields carry the names and
 * meaning of the reference's public state projection (csrc/engine.cu:3200-3211 STATE_FIELDS,
 * read by tests/test_engine.py:1666-1730): phase (0 free, 1 span, 2 escaped, 3 error),
 * pos (opener/closer bytes matched outside a span), segment (0 subject, 1 relation,
 * 2 object), depth, [lo, hi) the typed label's row range (-1 when the label branch is
 * dead), the closer/separator branches' bytes matched and the label rows they started
 * after, the escape branch's bytes matched, the candidate subject and relation rows,
 * subj_key (first row of the subject label), hops (relations of the open path, this one
 * included), four expression fields (the operator branch's bytes matched and the operator
 * they fit, the span's operator 1..3 or 0, the operand being written: 0 A, 1 B), the
 * end-after-answer flag and the last closed span (kind 0 none, 1 unresolved, 2 entity,
 * 3 fact, 4 path, 5 comparison, 6 relation plan; its rows; a comparison, as the
 * reference engine records it: last_lo / last_hi the label rows of the operands' committed
 * starts, last_subj_lo the result: 0 A, 1 B, 2 both, 3 the verdict yes, 4 no, last_subj_hi
 * the operator).  ex_hi and flags are this engine's own: the end of the
 * typed label's exact rows and which delimiter branches may start next (or that STOP
 * holds); stop_used_lo/hi are the reference's STOP mask (csrc/engine.cu:88). */
typedef struct XgState {
  int32_t phase, pos, segment, depth, lo, hi;
  int32_t close_pos, close_lo, close_hi;
  int32_t sep_pos, sep_lo, sep_hi;
  int32_t esc_pos;
  int32_t subj_lo, subj_hi, rel_lo, rel_hi, subj_key, hops;
  int32_t op_pos, op_kind, op, operand;
  int32_t answer_complete;
  int32_t last_kind, last_lo, last_hi, last_subj_lo, last_subj_hi, last_rel_lo, last_rel_hi;
  int32_t ex_hi, flags;
  int32_t stop_used_lo, stop_used_hi;  /* residual-goal STOP: question words the path has used (64-bit mask) */
  int32_t reserved[29];
} XgState;

#define XG_STATE_INTS 64

/* Where each table lives in the packed index blob: byte offsets (16-byte aligned; -1 for
 * an absent optional table) and the sizes the kernels need.  Built by the host-side
 * table packer (xgraph_b200/tables.py, the counterpart of src/xgraph/engine.py:311-556
 * native_tables). */
typedef struct XgLayout {
  int64_t blob_bytes;
  int32_t vocab, words, words_padded;
  int32_t entity_rows, relation_rows, entities, relations, relation_words;
  int32_t opener_len, closer_len, separator_len, escape_len;
  int32_t versions, wide_count;
  int32_t ent_cols, rel_cols;  /* depths stored column-major in ent_col / rel_col */
  int32_t pad0, pad1;
  int64_t ent_tok, ent_off, ent_owner, rel_tok, rel_off, rel_owner;
  int64_t ent_col, rel_col;      /* int32 [cols][rows]: token at depth d of each row, -1 past its end */
  int64_t ent_first, rel_first;  /* int32 [vocab + 1]: first row whose first token is >= t */
  int64_t ent_first_row, ent_rows_off, ent_rows;
  int64_t adj_off, edge_rel, edge_obj;
  int64_t sitelinks, kept_prefix;
  int64_t root_mask, wide_keys, wide_masks;
  int64_t free_next, free_mask, esc_next, esc_mask, eos_mask;
  int64_t closer_off, closer_tok, closer_next;
  int64_t separator_off, separator_tok, separator_next;
  int64_t escape_off, escape_tok, escape_next;
  int64_t ver_off, ver_subj, ver_adj, ver_edge_rel, ver_edge_obj;
  int64_t dstep;  /* uint64 [vocab]: packed next positions of every delimiter byte position, or -1 */
  int64_t row_degree;  /* int32 [entity_rows]: base-KG adjacency entries of each label row's owner */
  int64_t row_first;   /* int32 [entity_rows]: first label row of each label row's owner */
  int64_t run_off;     /* int32 [entities + 1]: each entity's relation runs in `runs` (CSR) */
  int64_t runs;        /* int32 [runs + 1][2]: (relation, first edge) of each run of equal relations in an
                          entity's adjacency; the last pair (INT32_MAX, edges) closes the final run */
  int64_t run_rel;     /* int32 [runs]: the relation of each run (the first column of `runs`) */
  int64_t edge_first;  /* int32 [edges]: first label row of each edge's object entity, bit 31 set when
                          that entity has no triples in the base KG */
  int64_t row_sitelinks; /* int32 [entity_rows]: sitelinks of each label row's owner, or -1 */
} XgLayout;

/* Span-language policies, as the reference Engine's constructor flags
 * (src/xgraph/engine.py:582-623).  Observation, menu and audit policies are not part of
 * this engine (residual-goal STOP: xg_enable_stop).
 *
 * The logit policies of apply_mask (and of the sync_apply steps, which include it), as the
 * native Engine's arguments (csrc/engine.cu:2601, 2668-2671):
 *   release_log_mass  log of the release mass (< 0), -INFINITY when off: inside a span, a
 *                     row whose logits put less than exp(release_log_mass) of their softmax
 *                     (over the served vocabulary, at the logits' own temperature) on the
 *                     allowed set may write only the escape marker's next tokens;
 *   release_top       1: the same for a row whose own top token (lowest column among
 *                     equal maxima) is disallowed;
 *   escape_bias       added to the logits of the tokens that commit to the escape marker
 *                     inside a span (they start it and continue neither the label, the
 *                     separator nor the closer); 0 when off.  16-bit logits hold the sum
 *                     rounded to nearest.
 * Release needs escapes.  A released row's mask is used for that call only: the slot's
 * recorded mask (xg_fill_mask, xg_mask_host) is the ordinary one. */
typedef struct XgOptions {
  int32_t escapes, repeats, derivation, paths, bound_escapes, committed_paths;
  int32_t sitelinks_rank, end_after_answer;
  int32_t release_top;
  float release_log_mass, escape_bias;
  /* relation support of path mode's relation segments, as the reference Engine's
   * `relations` (src/xgraph/engine.py:666-668, csrc/engine.cu:354): 0 frontier (paths
   * execute), 1 vocabulary (every relation), 2 successor (after the first relation, the
   * successors of the preceding label's relations; tables from
   * xg_set_relation_successors).  1 and 2 need path mode and no STOP; a closed plan is
   * unresolved (last_kind 6) and binds nothing. */
  int32_t relations;
  /* 1: expressions, the date and value comparisons, as the reference Engine's
   * `expressions` (src/xgraph/engine.py:655-664, csrc/engine.cu:374-391): a span may be
   * `⟦ earlier: A | B · r⟧` (or later:, same:); needs committed paths, escapes and frontier
   * support, and its tables from xg_set_expressions before the first sync.  Each slot's
   * memory then holds an operand region after its relation bitmap. */
  int32_t expressions;
} XgOptions;

typedef struct XgInfo {
  int32_t max_sequences, vocab, words, words_padded, memory_ints, device;
} XgInfo;

/* One request's admission into a slot, applied in the reference adapter's order
 * (src/xgraph/vllm.py:569-605 apply_staged_writes): begin (on = 1) or end (on = 0), then the
 * anchor rows (derivation / path mode: sorted, distinct label rows; the first 64 count),
 * then the KG version (0 = base), then open_span.  Field meanings are those of
 * Engine::begin, set_reached, set_version and open_span (csrc/engine.cu:2818-2876, 2955). */
#define XG_MAX_ANCHORS 64
typedef struct XgAdmission {
  int32_t slot;
  int32_t on;
  int32_t version;
  int32_t open_span;
  int32_t anchor_count;
  int32_t anchors[XG_MAX_ANCHORS];
} XgAdmission;

typedef struct XgEngine XgEngine;

/* Message of this thread's last failed call ("" if none). */
XG_API const char* xg_last_error(void);
XG_API int32_t xg_abi_version(void);

/* Engine(tables, vocab, words, max_sequences, ...) (csrc/engine.cu:2600-2797): copy the
 * packed index blob (host memory) to the current device and allocate max_sequences slots,
 * all inactive in the initial state. */
XG_API int xg_create(const void* blob_host, const XgLayout* layout, const XgOptions* options,
              int32_t max_sequences, XgEngine** out);
/* As xg_create from a blob already on the current device (for example one received by an
 * NCCL broadcast); the engine copies it and does not keep the caller's pointer. */
XG_API int xg_create_from_device(const void* blob_device, const XgLayout* layout,
                          const XgOptions* options, int32_t max_sequences, XgEngine** out);
XG_API int xg_destroy(XgEngine* engine);
XG_API int xg_info(const XgEngine* engine, XgInfo* out);

/* Engine::reset (csrc/engine.cu:2799-2814): every slot inactive, initial state. */
XG_API int xg_reset(XgEngine* engine, void* stream);
/* Engine::begin (csrc/engine.cu:2818-2826): slots (device int32[count]) back to the
 * initial state, base KG, cursor unset; active = on. */
XG_API int xg_begin(XgEngine* engine, const int32_t* slots, int32_t count, int32_t on, void* stream);
/* Engine::set_reached (csrc/engine.cu:2840-2860): anchor rows (host int32, sorted; the
 * first 64 are kept). */
XG_API int xg_set_reached(XgEngine* engine, int32_t slot, const int32_t* rows, int32_t count, void* stream);
/* Register one KG version while the engine runs (no blob rebuild); the reference registers
 * versions only when an engine is built (src/xgraph/engine.py versions=, csrc/engine.cu:
 * 477-491 reads them), with the same layout per version (src/xgraph/kgversions.py:14-21,
 * 203-303): `count` sorted edited subjects (entity positions), each with its whole edge
 * list in the new version, edges subjects' adjacency[i] .. adjacency[i + 1] (adjacency:
 * count + 1 offsets from 0) of edge_relations / edge_objects (relation positions, object
 * label rows), sorted by (relation, object row).  Host arrays, checked, then copied into the
 * engine's version arena on `stream` (which grows, and frees its old buffers in stream
 * order, when full).  *version receives the number slots select with xg_set_version or an
 * admission: the lowest number a dropped version left free, else the next one.  Calls that
 * add or drop versions must be ordered with the engine's kernels (one stream). */
XG_API int xg_add_version(XgEngine* engine, const int32_t* subjects, int32_t count, const int64_t* adjacency,
                          const int32_t* edge_relations, const int32_t* edge_objects, void* stream,
                          int32_t* version);
/* Forget a registered version: slots still selecting it read the base KG from the next launch
 * on; its number is reused by a later xg_add_version. */
XG_API int xg_drop_version(XgEngine* engine, int32_t version, void* stream);
/* Engine::set_version (csrc/engine.cu:2864-2876): 0 = base KG, else a registered version. */
XG_API int xg_set_version(XgEngine* engine, int32_t slot, int32_t version, void* stream);
/* Engine::open_span (csrc/engine.cu:2955-2962): the slot starts inside a span. */
XG_API int xg_open_span(XgEngine* engine, int32_t slot, void* stream);
/* Residual-goal STOP (the reference engine's stop="residual-goal", csrc/engine.cu:1001-1072,
 * 1580-1583, 1872, 1902): enable it on an engine (path mode with committed paths) with the
 * case-folded words of every entity label row, host CSR: label_offsets int64 [entity_rows
 * + 1] into label_words, each row's words (its text after the label prefix, \w+ runs,
 * case-folded) each followed by a 0 byte.  Allocates the per-slot STOP tables; slots start
 * without one. */
XG_API int xg_enable_stop(XgEngine* engine, const int64_t* label_offsets, const uint8_t* label_words,
                          int64_t word_bytes);
/* Engine::set_stop (csrc/engine.cu:2909-2940): one request's STOP table for the slot, host
 * arrays: relations int32 [relation_count][3] (per relation number: 1 when the question's
 * answer head names it, then the 64-bit mask of the relevant question words it covers, low
 * and high halves), the relevant question words' UTF-8 bytes (at most 4096) and their
 * offsets int32 [count + 1] (from 0 to word_bytes, count at most 64).  Call after begin; the
 * slot's next begin (or admission) clears it.  XG_EINVAL without xg_enable_stop. */
XG_API int xg_set_stop(XgEngine* engine, int32_t slot, const int32_t* relations, int32_t relation_count,
                       const uint8_t* words, int32_t word_bytes, const int32_t* offsets, int32_t offset_count,
                       void* stream);
/* The successor tables of successor support (the reference engine's native table
 * "relation_successors", src/xgraph/relations.py:31-60, csrc/engine.cu:355, 2734), host
 * uint32 [tables][relations][relation_words]: table v (0 the base KG, then the versions
 * built into the engine in order), bit r2 of row r1 set when some object of an r1 edge is
 * the subject of an r2 edge in that KG.  Copied to the device (synchronously) before the
 * first step; XG_EINVAL unless the engine was created with relations = 2, with more than
 * 10,304 relations, or with fewer tables than 1 + the built-in versions. */
XG_API int xg_set_relation_successors(XgEngine* engine, const uint32_t* tables, int32_t table_count);
/* The expression tables (the reference engine's native tables operand_*, operator<k>_*,
 * operator_lcp, date_entities / date_lo / date_hi / date_keys and verdict_entities,
 * src/xgraph/engine.py:345-360, 500-530, csrc/engine.cu:2745-2792), from host memory:
 *   delimiters      int32 [delimiter_ints]: the operand separator's token lists, then each
 *                   offered operator's (written after the label prefix, so with it in
 *                   front), one after another, each as its length L (1..64), its L + 1 CSR
 *                   offsets over byte positions, its tokens (ascending per position) and
 *                   each token's next byte position (L: the delimiter complete);
 *   operators       how many operators are offered (1..4; the value comparison, the third,
 *                   only with the verdict entities);
 *   operator_lcp    int32 [operators][operators]: the leading bytes two operators share;
 *   date_entities   int32 [dates]: the date entities' positions, ascending;
 *   date_keys       int32 [dates]: their dates, packed (year << 11 | month << 7 | day << 2 |
 *                   precision; 0 for an unstated month or day);
 *   verdicts        int32 [2]: the verdict entities' positions (yes, no), or null.
 * Copied to the device (synchronously) before the first step; XG_EINVAL unless the engine
 * was created with expressions = 1, or for malformed tables. */
XG_API int xg_set_expressions(XgEngine* engine, const int32_t* delimiters, int64_t delimiter_ints, int32_t operators,
                              const int32_t* operator_lcp, const int32_t* date_entities, const int32_t* date_keys,
                              int32_t dates, const int32_t* verdicts);
/* Engine::advance (csrc/engine.cu:3041-3054): advance slots 0..count-1 by tokens[i];
 * tokens_on_host != 0 means host memory (copied first). */
XG_API int xg_advance(XgEngine* engine, const int32_t* tokens, int32_t count, int32_t tokens_on_host,
               void* stream);
/* Engine::sync (csrc/engine.cu:2966-2985): each listed active slot advances over
 * history[slot * history_stride + cursor .. total_len[slot]) (cursor = prompt_len[slot]
 * the first time); history, prompt_len and total_len are device (or pinned host)
 * memory with one row / entry per slot (history_rows and lengths_count >= max_sequences). */
XG_API int xg_sync(XgEngine* engine, const int32_t* slots, int32_t count, const int32_t* history,
            int64_t history_stride, int64_t history_rows, const int32_t* prompt_len,
            const int32_t* total_len, int64_t lengths_count, void* stream);
/* Engine::fill_mask (csrc/engine.cu:3056-3062): materialize the masks of slots
 * 0..sequences-1 into the mask buffer. */
XG_API int xg_fill_mask(XgEngine* engine, int32_t sequences, void* stream);
/* Engine::mask: the device mask buffer, max_sequences rows of words_padded uint32. */
XG_API int xg_mask_device(XgEngine* engine, uint32_t** out);
/* The device state array, max_sequences XgState records (read-only for callers; no
 * reference counterpart beyond states_host, which copies it). */
XG_API int xg_states_device(XgEngine* engine, XgState** out);
/* Engine::mask_host / states_host (csrc/engine.cu:3076-3084): wait for the device, then
 * copy sequences x words mask words / sequences x XG_STATE_INTS state words. */
XG_API int xg_mask_host(XgEngine* engine, int32_t sequences, uint32_t* out);
XG_API int xg_states_host(XgEngine* engine, int32_t sequences, int32_t* out);
/* Diagnostic: wait, then copy the slots' memory (facts, reached rows, frontier, version). */
XG_API int xg_memory_host(XgEngine* engine, int32_t sequences, int32_t* out);
/* sync then apply_mask in one launch, for a step without speculative draft rows: logits row
 * i belongs to slots[i] (rows x cols, row_stride elements apart); the other arguments are
 * xg_sync's.  Same results as xg_sync followed by xg_apply_mask with row_slots = slots.
 * The reference has no fused call (its adapter calls sync, then apply_mask). */
XG_API int xg_sync_apply(XgEngine* engine, const int32_t* slots, int32_t count, const int32_t* history,
                         int64_t history_stride, int64_t history_rows, const int32_t* prompt_len,
                         const int32_t* total_len, int64_t lengths_count, void* logits, int32_t dtype,
                         int32_t cols, int64_t row_stride, void* stream);
/* xg_sync_apply with the step's admissions folded into the same launch: admissions[0 ..
 * admit_count) (distinct slots; host memory when admissions_on_host != 0, else device
 * memory) are applied first, exactly as xg_admit would, then every listed slot syncs and
 * its logits row is masked.  One launch per decoding step whether or not requests join.
 * The reference's adapter reaches the same state with begin / set_reached / set_version /
 * open_span calls before sync (src/xgraph/vllm.py:569-631).  Host admissions are copied
 * into an engine buffer on `stream` (calls on one engine must be ordered on one stream);
 * device admissions with a field out of range are skipped and counted by xg_faults. */
XG_API int xg_sync_apply_admit(XgEngine* engine, const int32_t* slots, int32_t count, const int32_t* history,
                               int64_t history_stride, int64_t history_rows, const int32_t* prompt_len,
                               const int32_t* total_len, int64_t lengths_count, void* logits, int32_t dtype,
                               int32_t cols, int64_t row_stride, const XgAdmission* admissions,
                               int32_t admit_count, int32_t admissions_on_host, void* stream);
/* One launch for a batch of admissions (the reference's apply_staged_writes loop of begin,
 * set_reached, set_version and open_span calls, one launch per slot and op each): applies
 * admissions[0 .. count) (distinct slots; host memory when on_host != 0) and rebuilds
 * each admitted slot's mask. */
XG_API int xg_admit(XgEngine* engine, const XgAdmission* admissions, int32_t count, int32_t on_host, void* stream);
/* Device-side faults recorded since the last call, then cleared (waits for the device):
 * bit 1 (value 2) a device admission with a field out of range was skipped; bit 2 (value
 * 4) a fused step wrote a row's columns outside the relation-segment superset early and
 * the row then left its relation segment (its -inf would be wrong; never expected: the
 * early-write rule follows the state machine's own branches).  Bit 0 is unused.  0 in
 * normal operation. */
XG_API int xg_faults(XgEngine* engine, int32_t* out);
/* Engine::apply_mask (csrc/engine.cu:2990-3037): in place, logits[r, c] = -inf for every
 * column c its slot's mask disallows and every c >= vocab; rows of inactive slots and of
 * slots in the error phase are left untouched.  logits: device, dtype XG_F32/XG_BF16/XG_F16,
 * rows x cols with row_stride elements between rows.  row_slots: device int32[rows].
 * local_pos/input_ids: device int32[rows] for speculative draft rows, or both NULL.  With
 * draft rows (csrc/engine.cu:2353-2360), row r at offset k = local_pos[r] of its request's
 * rows is masked as if input_ids[r - k + 1 .. r] had been committed to its slot, whose state
 * does not move; a row whose drafts reach the error phase, or with k < 0 or k > r, is left
 * untouched.  The engine keeps scratch for the largest row count seen (memory and mask rows,
 * about 4 * (words + 600) bytes per row), allocated on the first call with more rows, after
 * synchronizing `stream`. */
XG_API int xg_apply_mask(XgEngine* engine, void* logits, int32_t dtype, int32_t rows, int32_t cols,
                  int64_t row_stride, const int32_t* row_slots, const int32_t* local_pos,
                  const int32_t* input_ids, void* stream);
/* No counterpart in the reference: xg_apply_mask for draft rows (local_pos and input_ids
 * required) that allocates nothing, for callers that may not allocate device memory while
 * they decode (a serving loop whose framework has already claimed the free memory for its
 * own pools, or code that must not take the synchronizing growth path of xg_apply_mask).
 * Its scratch is one static 8 MiB device array in this library, which every GPU that loads
 * the library holds until the process exits, shared by every call on the device: a call
 * with more rows than fit (4 * (words + 600) bytes per row) fails with XG_EINVAL and
 * launches nothing.  The array keeps the last call's contents; no part of it needs to
 * start at zero (each row's memory copy and mask row is written before it is read).  Calls whose kernels overlap on
 * the GPU (other streams, other engines, other threads) race on the array: order them.
 * The first call on a device looks the array's address up (cudaGetSymbolAddress, with the
 * engine's device current), which may also load the library's device code; make that first
 * call before any stream capture.  The address is kept for the life of the process: after a
 * cudaDeviceReset (which destroys the context holding the array) the process must reload the
 * library before it calls this function again.  Same results as xg_apply_mask with the same
 * arguments. */
XG_API int xg_apply_mask_noalloc(XgEngine* engine, void* logits, int32_t dtype, int32_t rows, int32_t cols,
                                 int64_t row_stride, const int32_t* row_slots, const int32_t* local_pos,
                                 const int32_t* input_ids, void* stream);

/* Device-side build of a KG index's adjacency; it replaces the host build of the same
 * arrays (src/xgraph/index.py:403-516, whose edge step turns every position triple into
 * one edge per label row of its object, deduplicated and sorted by (subject, relation,
 * object row)).  All arrays are device memory: triples as three int32 position arrays of
 * length `triples`; the entities' label rows as CSR (row_offsets int64 [entities + 1],
 * row_list int32: each entity's label rows in row order); writable uint8 [relation_count]
 * (1 where the relation has a relation label row).  A triple is writable when its subject
 * and object have label rows and its relation is writable; *unwritable counts the others.
 * Called with offsets == NULL it only sizes: *edges = the edge count before
 * deduplication, the capacity the edge arrays need.  Called with offsets int64
 * [entities + 1] and edge_relations / edge_objects int32 [capacity], it writes the CSR
 * and *edges = the edge count.  A position out of range fails with XG_EINVAL.  Device
 * scratch is allocated and freed on `stream` (stream-ordered); the call synchronizes the
 * stream before it returns. */
XG_API int xg_build_adjacency(const int32_t* subjects, const int32_t* relations, const int32_t* objects,
                              int64_t triples, const int64_t* row_offsets, const int32_t* row_list, int32_t entities,
                              int32_t label_rows, const uint8_t* writable, int32_t relation_count, int64_t capacity,
                              int64_t* offsets, int32_t* edge_relations, int32_t* edge_objects, int64_t* edges,
                              int64_t* unwritable, void* stream);

/* Device-side label rows of a KG index; it replaces the host build of the same arrays
 * (src/xgraph/index.py:167-233: every label, written as label prefix + label and encoded by
 * the served tokenizer, is admitted under exact-v1 -- no special token, a nonempty
 * encoding, known bytes for every token, and token bytes equal to the written bytes -- and
 * the admitted labels become rows sorted as (token sequence, owner position) tuples).
 * Device arrays: label i's token ids token_ids[token_off[i] .. token_off[i + 1]) (token_off
 * int64 [labels + 1], token_ids int32 [token_count]), its written bytes
 * text[text_off[i] .. text_off[i + 1]) (text_off int64 [labels + 1], text uint8
 * [text_bytes]), its owner position owners[i] in [0, owner_count); the served vocabulary's
 * bytes as CSR over `vocab` ids (vocab_off int64 [vocab + 1], vocab_bytes uint8
 * [vocab_byte_count]) with vocab_kind int8 [vocab] (0 known bytes, 1 special, 2 unknown
 * bytes; ids outside [0, vocab) have unknown bytes).  Outputs: status int32 [labels] (0
 * admitted, 1 a special token, 2 an empty encoding, 3 a token with unknown bytes, 4 the
 * bytes do not round-trip: the reference's checks in its order), row_offsets int64
 * [labels + 1], row_tokens int32 [token_count] and row_owners int32 [labels] for the
 * first *rows rows (*tokens tokens), host outputs.  Offsets outside their arrays or an owner
 * out of range fail with XG_EINVAL.  Scratch is stream-ordered on `stream`; the call
 * synchronizes the stream before it returns. */
XG_API int xg_build_label_rows(int32_t labels, const int64_t* token_off, const int32_t* token_ids,
                               int64_t token_count, const int64_t* text_off, const uint8_t* text,
                               int64_t text_bytes, const int32_t* owners, int32_t owner_count,
                               int32_t vocab, const int64_t* vocab_off, const uint8_t* vocab_bytes,
                               int64_t vocab_byte_count, const int8_t* vocab_kind, int32_t* status,
                               int64_t* row_offsets, int32_t* row_tokens, int32_t* row_owners,
                               int32_t* rows, int64_t* tokens, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* XGRAPH_B200_H */
