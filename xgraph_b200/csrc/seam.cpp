// Host test seam: the engine's per-row logic (core.cuh) compiled as sequential C++.
//
// TEST ONLY.  tests/seam.py builds this file with g++ and replays oracle walks through it
// on the CPU, so logic errors in core.cuh show up without a GPU.  The product library
// (libxgraph_b200.so, engine.cu) never loads or links it, and it exports xgs_* names that
// nothing in xgraph_b200/ calls.
#include <cstring>
#include <vector>

#include "core.cuh"

using namespace xg;

struct SeamEngine {
  std::vector<char> blob;
  XgLayout layout{};
  int32_t slots = 0;
  std::vector<XgState> states;
  std::vector<int32_t> memory;
  std::vector<uint32_t> masks;
  std::vector<const uint32_t*> base;
  std::vector<uint32_t*> delta;
  std::vector<int32_t> cursors, active;
  std::vector<Key> top;
  std::vector<int32_t> scratch;
  std::vector<int32_t> ver_range;  // the blob's cumulative version offsets as (begin, end) pairs
  // residual-goal STOP (xgs_enable_stop)
  std::vector<int64_t> stop_label_off;
  std::vector<uint8_t> stop_label_words;
  std::vector<int32_t> stop_on, stop_rel, stop_woff;
  std::vector<uint8_t> stop_words;
  std::vector<uint32_t> successors;  // successor support's tables (xgs_set_successors)
  // expressions (xgs_set_expressions): the packed delimiter lists, the date table
  std::vector<int32_t> expr_delims, date_entities, date_keys, date_lo, date_hi;
  Tables t{};
};

template <class T>
static const T* at(const char* blob, int64_t offset) {
  return offset < 0 ? nullptr : reinterpret_cast<const T*>(blob + offset);
}

static Ctx ctx(SeamEngine* e, int32_t slot) {
  return Ctx{e->t, Warp{0}, slot, e->memory.data() + static_cast<int64_t>(slot) * e->t.memory_ints, e->top.data(),
             e->scratch.data()};
}

static void begin_slot(SeamEngine* e, int32_t slot, int32_t on) {
  std::memset(&e->states[slot], 0, sizeof(XgState));
  int32_t* mem = e->memory.data() + static_cast<int64_t>(slot) * e->t.memory_ints;
  mem[kMemFacts] = mem[kMemReached] = mem[kMemFrontier] = mem[kMemVersion] = 0;
  mem[kMemPendingLo] = -1;
  e->cursors[slot] = -1;
  e->active[slot] = on;
  e->base[slot] = e->t.free_mask;
  e->delta[slot] = nullptr;
  if (!e->stop_on.empty()) e->stop_on[slot] = 0;
}

extern "C" {

SeamEngine* xgs_create(const void* blob, const XgLayout* l, const XgOptions* o, int32_t slots) {
  SeamEngine* e = new SeamEngine();
  e->blob.assign(static_cast<const char*>(blob), static_cast<const char*>(blob) + l->blob_bytes);
  e->layout = *l;
  e->slots = slots;
  const char* b = e->blob.data();
  Tables& t = e->t;
  t.ent = Rows{at<int32_t>(b, l->ent_tok), at<int32_t>(b, l->ent_off), at<int32_t>(b, l->ent_owner), l->entity_rows,
               at<int32_t>(b, l->ent_col), at<int32_t>(b, l->ent_first), l->ent_cols};
  t.rel = Rows{at<int32_t>(b, l->rel_tok), at<int32_t>(b, l->rel_off), at<int32_t>(b, l->rel_owner), l->relation_rows,
               at<int32_t>(b, l->rel_col), at<int32_t>(b, l->rel_first), l->rel_cols};
  t.ent_first_row = at<int32_t>(b, l->ent_first_row);
  t.row_degree = at<int32_t>(b, l->row_degree);
  t.row_first = at<int32_t>(b, l->row_first);
  t.ent_rows_off = at<int32_t>(b, l->ent_rows_off);
  t.ent_rows = at<int32_t>(b, l->ent_rows);
  t.adj_off = at<int32_t>(b, l->adj_off);
  t.edge_rel = at<int32_t>(b, l->edge_rel);
  t.edge_obj = at<int32_t>(b, l->edge_obj);
  t.run_off = at<int32_t>(b, l->run_off);
  t.runs = at<int32_t>(b, l->runs);
  t.run_rel = at<int32_t>(b, l->run_rel);
  t.edge_first = at<int32_t>(b, l->edge_first);
  t.sitelinks = o->sitelinks_rank ? at<int32_t>(b, l->sitelinks) : nullptr;
  t.row_sitelinks = o->sitelinks_rank ? at<int32_t>(b, l->row_sitelinks) : nullptr;
  t.kept_prefix = at<int32_t>(b, l->kept_prefix);
  t.root_mask = at<uint32_t>(b, l->root_mask);
  t.wide_keys = at<int64_t>(b, l->wide_keys);
  t.wide_masks = at<uint32_t>(b, l->wide_masks);
  t.wide_count = l->wide_count;
  t.free_next = at<int8_t>(b, l->free_next);
  t.free_mask = at<uint32_t>(b, l->free_mask);
  t.esc_next = at<int8_t>(b, l->esc_next);
  t.esc_mask = at<uint32_t>(b, l->esc_mask);
  t.eos_mask = at<uint32_t>(b, l->eos_mask);
  t.closer = Delim{at<int32_t>(b, l->closer_off), at<int32_t>(b, l->closer_tok), at<int32_t>(b, l->closer_next), l->closer_len};
  t.separator = Delim{at<int32_t>(b, l->separator_off), at<int32_t>(b, l->separator_tok), at<int32_t>(b, l->separator_next),
                      l->separator_len};
  t.escape = Delim{at<int32_t>(b, l->escape_off), at<int32_t>(b, l->escape_tok), at<int32_t>(b, l->escape_next), l->escape_len};
  for (Delim* d : {&t.closer, &t.separator, &t.escape}) {
    for (int32_t k = 0; k < 17; ++k) d->at[k] = k <= d->len ? d->off[k] : 0;
  }
  t.dstep = at<uint64_t>(b, l->dstep);
  const int32_t* ver_off = at<int32_t>(b, l->ver_off);
  for (int32_t v = 0; v < l->versions; ++v) {
    e->ver_range.push_back(ver_off[v]);
    e->ver_range.push_back(ver_off[v + 1]);
  }
  e->ver_range.push_back(0);  // never empty
  t.ver_range = e->ver_range.data();
  t.ver_subj = at<int32_t>(b, l->ver_subj);
  t.ver_adj = at<int32_t>(b, l->ver_adj);
  t.ver_edge_rel = at<int32_t>(b, l->ver_edge_rel);
  t.ver_edge_obj = at<int32_t>(b, l->ver_edge_obj);
  t.versions = l->versions;
  t.vocab = l->vocab;
  t.words = l->words;
  t.words_padded = l->words_padded;
  t.entities = l->entities;
  t.relations = l->relations;
  t.relation_words = l->relation_words;
  t.escapes = o->escapes;
  t.repeats = o->repeats;
  t.derivation = o->derivation || o->paths;
  t.paths = o->paths;
  t.bound_escapes = o->bound_escapes;
  t.committed = o->committed_paths;
  t.end_after_answer = o->end_after_answer;
  t.relation_mode = o->relations;
  t.memory_ints = memory_ints_for(l->relation_words, o->expressions != 0);
  t.mem_operand = o->expressions ? memory_ints_for(l->relation_words, false) : 0;
  e->states.assign(slots, XgState{});
  e->memory.assign(static_cast<size_t>(slots) * t.memory_ints, 0);
  e->masks.assign(static_cast<size_t>(slots) * l->words_padded, 0u);
  e->base.assign(slots, nullptr);
  e->delta.assign(slots, nullptr);
  e->cursors.assign(slots, -1);
  e->active.assign(slots, 0);
  e->top.assign(kTopCap, Key{});
  e->scratch.assign(kScratchInts + 2, 0);
  t.states = e->states.data();
  t.memory = e->memory.data();
  t.masks = e->masks.data();
  t.base = e->base.data();
  t.delta = e->delta.data();
  t.cursors = e->cursors.data();
  t.active = e->active.data();
  for (int32_t s = 0; s < slots; ++s) begin_slot(e, s, 0);
  return e;
}

void xgs_destroy(SeamEngine* e) { delete e; }

void xgs_begin(SeamEngine* e, int32_t slot, int32_t on) { begin_slot(e, slot, on); }

void xgs_set_version(SeamEngine* e, int32_t slot, int32_t version) {
  Ctx c = ctx(e, slot);
  c.mem[kMemVersion] = version;
  c.mem[kMemPendingLo] = -1;
  XgState s = e->states[slot];
  if (s.phase == kSpan) set_flags(c, s);
  e->states[slot] = s;
  build_mask(c, s);
}

void xgs_set_reached(SeamEngine* e, int32_t slot, const int32_t* rows, int32_t count) {
  Ctx c = ctx(e, slot);
  if (count > kMaxSet) count = kMaxSet;
  for (int32_t i = 0; i < count; ++i) c.mem[kMemReachedRows + i] = rows[i];
  c.mem[kMemReached] = count;
  c.mem[kMemPendingLo] = -1;
  XgState s = e->states[slot];
  if (s.phase == kSpan) set_flags(c, s);
  e->states[slot] = s;
  build_mask(c, s);
}

void xgs_open_span(SeamEngine* e, int32_t slot) {
  Ctx c = ctx(e, slot);
  XgState s = e->states[slot];
  if (s.phase != kError) {
    s.answer_complete = 0;
    open_span(c, s);
  }
  e->states[slot] = s;
  build_mask(c, s);
}

void xgs_advance(SeamEngine* e, const int32_t* tokens, int32_t count) {
  for (int32_t slot = 0; slot < count; ++slot) {
    Ctx c = ctx(e, slot);
    XgState s = e->states[slot];
    advance_state(c, s, tokens[slot]);
    e->states[slot] = s;
    build_mask(c, s);
  }
}

// One slot advanced by one token (the other slots untouched).
void xgs_advance_slot(SeamEngine* e, int32_t slot, int32_t token) {
  Ctx c = ctx(e, slot);
  XgState s = e->states[slot];
  advance_state(c, s, token);
  e->states[slot] = s;
  build_mask(c, s);
}

// Masks of slots 0..n-1 as [n, words] (zeros for the error phase).
void xgs_masks(SeamEngine* e, int32_t n, uint32_t* out) {
  const int32_t words = e->layout.words;
  for (int32_t slot = 0; slot < n; ++slot) {
    const uint32_t* base = e->base[slot];
    const uint32_t* delta = e->delta[slot];
    for (int32_t w = 0; w < words; ++w)
      out[static_cast<int64_t>(slot) * words + w] = (base ? base[w] : 0u) | (delta ? delta[w] : 0u);
  }
}

void xgs_states(SeamEngine* e, int32_t n, int32_t* out) {
  std::memcpy(out, e->states.data(), static_cast<size_t>(n) * sizeof(XgState));
}

void xgs_memory(SeamEngine* e, int32_t n, int32_t* out) {
  std::memcpy(out, e->memory.data(), static_cast<size_t>(n) * e->t.memory_ints * sizeof(int32_t));
}

int32_t xgs_memory_ints(SeamEngine* e) { return e->t.memory_ints; }

// xg_set_expressions on the host (same arguments); 1 when the tables are malformed.
int32_t xgs_set_expressions(SeamEngine* e, const int32_t* delimiters, int64_t ints, int32_t operators,
                            const int32_t* lcp, const int32_t* date_entities, const int32_t* date_keys, int32_t dates,
                            const int32_t* verdicts) {
  Tables& t = e->t;
  PackedDelim parsed[1 + kMaxOperators];
  if (operators < 1 || operators > kMaxOperators || (operators > 2 && !verdicts) ||
      !parse_packed_delims(delimiters, ints, 1 + operators, t.vocab, parsed))
    return 1;
  e->expr_delims.assign(delimiters, delimiters + ints);
  const int32_t* base = e->expr_delims.data();
  for (int32_t k = 0; k <= operators; ++k) {
    Delim& d = k == 0 ? t.operand_sep : t.operators[k - 1];
    d = Delim{base + parsed[k].off, base + parsed[k].tok, base + parsed[k].next, parsed[k].len, {}};
    for (int32_t i = 0; i < 17; ++i) d.at[i] = parsed[k].at[i];
  }
  for (int32_t k = 0; k < kMaxOperators * kMaxOperators; ++k) t.operator_lcp[k] = 0;
  for (int32_t k = 0; k < operators; ++k)
    for (int32_t j = 0; j < operators; ++j) t.operator_lcp[k * kMaxOperators + j] = lcp[k * operators + j];
  e->date_entities.assign(date_entities, date_entities + dates);
  e->date_keys.assign(date_keys, date_keys + dates);
  e->date_lo.resize(dates);
  e->date_hi.resize(dates);
  for (int32_t i = 0; i < dates; ++i) {
    e->date_lo[i] = date_bound(date_keys[i], true);
    e->date_hi[i] = date_bound(date_keys[i], false);
  }
  t.date_entities = e->date_entities.data();
  t.date_keys = e->date_keys.data();
  t.date_lo = e->date_lo.data();
  t.date_hi = e->date_hi.data();
  t.date_count = dates;
  t.verdict_yes = verdicts ? verdicts[0] : -1;
  t.verdict_no = verdicts ? verdicts[1] : -1;
  t.operator_count = operators;
  return 0;
}

// xg_set_relation_successors on the host.
void xgs_set_successors(SeamEngine* e, const uint32_t* tables, int32_t count) {
  e->successors.assign(tables, tables + static_cast<size_t>(count) * e->t.relations * e->t.relation_words);
  e->t.successors = e->successors.data();
  e->t.successor_tables = count;
}

// xg_enable_stop / xg_set_stop on the host (arguments checked by the library's entry points).

void xgs_enable_stop(SeamEngine* e, const int64_t* offsets, const uint8_t* words, int64_t bytes) {
  const int64_t rows = e->layout.entity_rows;
  e->stop_label_off.assign(offsets, offsets + rows + 1);
  e->stop_label_words.assign(words, words + bytes);
  e->stop_on.assign(e->slots, 0);
  e->stop_rel.assign(static_cast<size_t>(e->slots) * e->t.relations * 3, 0);
  e->stop_woff.assign(static_cast<size_t>(e->slots) * (kMaxStopWords + 2), 0);
  e->stop_words.assign(static_cast<size_t>(e->slots) * kMaxStopBytes, 0);
  e->t.stop_label_off = e->stop_label_off.data();
  e->t.stop_label_words = e->stop_label_words.data();
  e->t.stop_on = e->stop_on.data();
  e->t.stop_rel = e->stop_rel.data();
  e->t.stop_woff = e->stop_woff.data();
  e->t.stop_words = e->stop_words.data();
}

void xgs_set_stop(SeamEngine* e, int32_t slot, const int32_t* relations, const uint8_t* words, int32_t bytes,
                  const int32_t* offsets, int32_t offset_count) {
  std::memcpy(e->stop_rel.data() + static_cast<int64_t>(slot) * e->t.relations * 3, relations,
              static_cast<size_t>(e->t.relations) * 3 * sizeof(int32_t));
  int32_t* woff = e->stop_woff.data() + static_cast<int64_t>(slot) * (kMaxStopWords + 2);
  woff[0] = offset_count - 1;
  for (int32_t k = 0; k < offset_count; ++k) woff[k + 1] = offsets[k];
  if (bytes > 0) std::memcpy(e->stop_words.data() + static_cast<int64_t>(slot) * kMaxStopBytes, words, bytes);
  e->stop_on[slot] = 1;
}

// apply_mask's logit policies for a slot: returns its escape position (-1: release leaves
// it alone); the tokens that commit it to the escape marker go to commits[0 .. *count) and
// the escape marker's next tokens from that position (its released mask) to
// released[0 .. *released_count), each list cut at cap.
int32_t xgs_escape_policy(SeamEngine* e, int32_t slot, int32_t* commits, int32_t* count, int32_t* released,
                          int32_t* released_count, int32_t cap) {
  const Ctx c = ctx(e, slot);
  const XgState& s = e->states[slot];
  int32_t n = 0;
  for_each_escape_commit(c, s, [&](int32_t token) {
    if (n < cap) commits[n] = token;
    ++n;
  });
  *count = n;
  const int32_t pos = escape_position(e->t, s);
  n = 0;
  if (pos >= 0) {
    for (int32_t i = delim_begin(e->t.escape, pos); i < delim_end(e->t.escape, pos); ++i) {
      if (n < cap) released[n] = e->t.escape.tok[i];
      ++n;
    }
  }
  *released_count = n;
  return pos;
}

// The edge range [out[0], out[1]) of `relation` in entity's adjacency (relative to the
// entity's first edge) and out[2] = the adjacency length, in KG version `version`.
void xgs_relation_slice(SeamEngine* e, int32_t version, int32_t entity, int32_t relation, int32_t* out) {
  const Edges g = edges_of(e->t, version, entity);
  relation_slice(e->t, g, relation, out[0], out[1]);
  out[2] = g.n;
}

}  // extern "C"
