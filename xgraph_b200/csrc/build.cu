// Device-side build of a KG index's adjacency (CSR edges per subject entity).
//
// The reference builds the index on the host (src/xgraph/index.py:403-516: every
// position triple (subject, relation, object) becomes one edge per label row of its
// object, the edges are deduplicated and sorted by (subject, relation, object row), and
// the subjects' edge ranges become CSR offsets).  Here the same arrays come out of four
// device passes over the triples:
//   check    per triple: is it writable (the subject and the object have label rows, the
//            relation has a relation row) and how many edges it expands to;
//   expand   each writable triple's edges as packed 64-bit keys subject|relation|row, at
//            its exclusive-scan offset;
//   sort     an LSD radix sort of the keys over just the bits they use, then unique
//            (CUB, the toolkit's header library);
//   decode   each unique key back into its relation and object row, and the subjects'
//            edge counts, whose scan is the CSR offsets.
// The keys order exactly as (subject, relation, row) tuples because each field gets the
// bits its largest value needs, so the result is the host build's, array for array.
#include <cub/cub.cuh>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "xgraph_b200.h"

namespace xg {
namespace build {

constexpr int32_t kThreads = 256;

inline int32_t bits_for(int64_t count) {  // bits that hold every value in [0, count)
  int32_t b = 0;
  while (b < 62 && (int64_t{1} << b) < count) ++b;
  return b;
}

inline unsigned grid_for(int64_t n) {
  const int64_t blocks = (n + kThreads - 1) / kThreads;
  return static_cast<unsigned>(blocks < 1 ? 1 : blocks > 65535 * 16 ? 65535 * 16 : blocks);
}

// Per triple: the number of edges it expands to (its object's label rows when it is
// writable, else 0); out-of-range positions are counted in bad[0] (and read nothing
// else), non-writable triples in bad[1].
__global__ void check_kernel(const int32_t* subjects, const int32_t* relations, const int32_t* objects, int64_t n,
                             const int64_t* row_offsets, int32_t entities, const uint8_t* writable,
                             int32_t relation_count, int64_t* repeat, unsigned long long* bad) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t s = subjects[i], r = relations[i], o = objects[i];
    int64_t count = 0;
    if (s < 0 || s >= entities || o < 0 || o >= entities || r < 0 || r >= relation_count) {
      atomicAdd(bad, 1ull);
    } else {
      const bool ok = row_offsets[s + 1] > row_offsets[s] && writable[r] != 0;
      count = ok ? row_offsets[o + 1] - row_offsets[o] : 0;
      if (count == 0) atomicAdd(bad + 1, 1ull);
    }
    repeat[i] = count;
  }
}

__global__ void expand_kernel(const int32_t* subjects, const int32_t* relations, const int32_t* objects, int64_t n,
                              const int64_t* row_offsets, const int32_t* row_list, const int64_t* repeat,
                              const int64_t* at, int32_t relation_bits, int32_t row_bits, uint64_t* keys) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t count = repeat[i];
    if (count == 0) continue;
    const uint64_t head = ((static_cast<uint64_t>(subjects[i]) << relation_bits) | static_cast<uint32_t>(relations[i]))
                          << row_bits;
    const int32_t* rows = row_list + row_offsets[objects[i]];
    uint64_t* out = keys + at[i];
    for (int64_t j = 0; j < count; ++j) out[j] = head | static_cast<uint32_t>(rows[j]);
  }
}

__global__ void decode_kernel(const uint64_t* keys, const int64_t* count, int32_t relation_bits, int32_t row_bits,
                              int32_t* edge_relations, int32_t* edge_objects, unsigned long long* degree) {
  const int64_t n = *count;
  const uint64_t row_mask = (uint64_t{1} << row_bits) - 1, relation_mask = (uint64_t{1} << relation_bits) - 1;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint64_t k = keys[i];
    edge_objects[i] = static_cast<int32_t>(k & row_mask);
    edge_relations[i] = static_cast<int32_t>((k >> row_bits) & relation_mask);
    atomicAdd(degree + (k >> (row_bits + relation_bits)), 1ull);
  }
}

// ---------------------------------------------------------------------------------------
// Label rows (src/xgraph/index.py:167-233): exact-v1 admission of every encoded label, then
// the admitted labels ordered as (token sequence, owner position) tuples.
//   admit   one warp per label: a special token (status 1), an empty encoding (2), a token
//           without known bytes (3), else its tokens' bytes against the written label
//           (label prefix + label, UTF-8): 4 when they differ, 0 admitted; offsets or ids
//           outside their arrays count in bad and give status -1;
//   select  the admitted labels, in input order (CUB);
//   sort    LSD over stable radix sorts: by owner, then by the token at each depth from the
//           deepest to the first, where a label already ended sorts first (key 0), as a
//           shorter tuple sorts before its extensions;
//   gather  each row's length, scanned into offsets, then its tokens and owner.

// Bytes class of each vocabulary id: 0 known bytes, 1 special, 2 unknown bytes.
constexpr int8_t kKnownBytes = 0, kSpecial = 1, kUnknownBytes = 2;

__global__ void admit_labels_kernel(int32_t labels, const int64_t* token_off, const int32_t* ids, int64_t id_count,
                                    const int64_t* text_off, const uint8_t* text, int64_t text_bytes,
                                    const int32_t* owners, int32_t owner_count, int32_t vocab,
                                    const int64_t* vocab_off, const uint8_t* vocab_bytes, int64_t vocab_byte_count,
                                    const int8_t* vocab_kind, int32_t* status, int32_t* selected, uint8_t* admitted,
                                    int32_t* length, unsigned long long* bad) {
  const int32_t lane = threadIdx.x & 31;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t i = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; i < labels; i += warps) {
    const int64_t t0 = token_off[i], t1 = token_off[i + 1], b0 = text_off[i], b1 = text_off[i + 1];
    const int32_t owner = owners[i];
    int32_t code = 0;
    if (t0 < 0 || t1 < t0 || t1 > id_count || b0 < 0 || b1 < b0 || b1 > text_bytes || owner < 0 ||
        owner >= owner_count) {
      code = -1;
    } else {
      bool special = false, unknown = false, broken = false;
      long long bytes = 0;
      for (int64_t j = t0 + lane; j < t1; j += 32) {
        const int32_t id = ids[j];
        const int8_t kind = id >= 0 && id < vocab ? vocab_kind[id] : kUnknownBytes;
        special |= kind == kSpecial;
        unknown |= kind == kUnknownBytes;
        if (kind == kKnownBytes) {
          const int64_t v0 = vocab_off[id], v1 = vocab_off[id + 1];
          broken |= v0 < 0 || v1 < v0 || v1 > vocab_byte_count;
          bytes += v1 - v0;
        }
      }
      special = __any_sync(0xffffffffu, special);
      unknown = __any_sync(0xffffffffu, unknown);
      broken = __any_sync(0xffffffffu, broken);
      for (int32_t d = 16; d > 0; d >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, d);
      code = special ? 1 : t1 == t0 ? 2 : unknown ? 3 : broken ? -1 : bytes != b1 - b0 ? 4 : 0;
      // the bytes, token by token (the loop is warp-uniform), lanes over each token's bytes
      int64_t at = b0;
      for (int64_t j = t0; j < t1 && code == 0; ++j) {
        const int32_t id = ids[j];
        const int64_t v0 = vocab_off[id], n = vocab_off[id + 1] - v0;
        bool differ = false;
        for (int64_t k = lane; k < n; k += 32) differ |= vocab_bytes[v0 + k] != text[at + k];
        if (__any_sync(0xffffffffu, differ)) code = 4;
        at += n;
      }
    }
    if (lane == 0) {
      status[i] = code;
      selected[i] = static_cast<int32_t>(i);
      admitted[i] = code == 0;
      length[i] = code == 0 ? static_cast<int32_t>(t1 - t0) : 0;
      if (code < 0) atomicAdd(bad, 1ull);
    }
  }
}

// keys[k] for sorted position k of the admitted labels: the owner (depth < 0), or the token
// at `depth` plus one (0 where the label has ended).
__global__ void label_keys_kernel(const int32_t* order, const int64_t* count, const int64_t* token_off,
                                  const int32_t* ids, const int32_t* owners, int32_t depth, uint32_t* keys) {
  const int64_t n = *count;
  for (int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; k < n;
       k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t i = order[k];
    if (depth < 0) {
      keys[k] = static_cast<uint32_t>(owners[i]);
    } else {
      const int64_t at = token_off[i] + depth;
      keys[k] = at < token_off[i + 1] ? static_cast<uint32_t>(ids[at]) + 1u : 0u;
    }
  }
}

__global__ void row_lengths_kernel(const int32_t* order, const int64_t* count, const int64_t* token_off,
                                   const int32_t* owners, int64_t* lengths, int32_t* row_owners) {
  const int64_t n = *count;
  for (int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; k < n;
       k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t i = order[k];
    lengths[k] = token_off[i + 1] - token_off[i];
    row_owners[k] = owners[i];
  }
}

// One warp per row: its tokens to their place in the row-ordered token array.
__global__ void row_tokens_kernel(const int32_t* order, const int64_t* count, const int64_t* token_off,
                                  const int32_t* ids, const int64_t* row_offsets, int32_t* row_tokens) {
  const int64_t n = *count;
  const int32_t lane = threadIdx.x & 31;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t k = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; k < n; k += warps) {
    const int32_t i = order[k];
    const int64_t from = token_off[i], len = token_off[i + 1] - from, to = row_offsets[k];
    for (int64_t j = lane; j < len; j += 32) row_tokens[to + j] = ids[from + j];
  }
}

}  // namespace build
}  // namespace xg

using namespace xg::build;

// Errors of this file go through xg_last_error like the engine's: the engine's file
// provides the setter.
extern "C" int xg_set_error(int code, const char* message);

namespace {

struct Scratch {  // stream-ordered device allocations, released on every return path
  cudaStream_t stream;
  void* held[12] = {};
  int n = 0;
  explicit Scratch(cudaStream_t s) : stream(s) {}
  template <class T>
  cudaError_t get(T** p, size_t bytes) {
    *p = nullptr;
    if (n == static_cast<int>(sizeof(held) / sizeof(held[0]))) return cudaErrorMemoryAllocation;  // table full
    void* q = nullptr;
    const cudaError_t e = cudaMallocAsync(&q, bytes ? bytes : 1, stream);
    if (e == cudaSuccess) held[n++] = q;
    *p = static_cast<T*>(q);
    return e;
  }
  ~Scratch() {
    for (int i = 0; i < n; ++i) cudaFreeAsync(held[i], stream);
  }
};

int build_fail(int code, const std::string& message) { return xg_set_error(code, message.c_str()); }

int build_cuda(cudaError_t e, const char* what) {
  cudaGetLastError();  // clear a non-sticky error so the next call starts clean
  return build_fail(XG_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

#define XG_BUILD_CUDA(call, what)                       \
  do {                                                  \
    const cudaError_t e_ = (call);                      \
    if (e_ != cudaSuccess) return build_cuda(e_, what); \
  } while (0)

extern "C" XG_API int xg_build_adjacency(const int32_t* subjects, const int32_t* relations, const int32_t* objects,
                                         int64_t triples, const int64_t* row_offsets, const int32_t* row_list,
                                         int32_t entities, int32_t label_rows, const uint8_t* writable,
                                         int32_t relation_count, int64_t capacity, int64_t* offsets,
                                         int32_t* edge_relations, int32_t* edge_objects, int64_t* edges,
                                         int64_t* unwritable, void* stream) {
  if (!edges || !unwritable) return build_fail(XG_EINVAL, "null edges or unwritable output");
  if (triples < 0 || entities < 0 || label_rows < 0 || relation_count < 0 || capacity < 0)
    return build_fail(XG_EINVAL, "negative size");
  if (triples > 0 && (!subjects || !relations || !objects)) return build_fail(XG_EINVAL, "null triples");
  if (!row_offsets || (label_rows > 0 && !row_list) || (relation_count > 0 && !writable))
    return build_fail(XG_EINVAL, "null label rows or writable flags");
  const int32_t subject_bits = bits_for(entities), relation_bits = bits_for(relation_count),
                row_bits = bits_for(label_rows);
  if (subject_bits + relation_bits + row_bits > 64) return build_fail(XG_EINVAL, "index too large for 64-bit edge keys");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  Scratch scratch(s);
  int64_t *repeat = nullptr, *at = nullptr, *count = nullptr;
  unsigned long long* bad = nullptr;
  XG_BUILD_CUDA(scratch.get(&repeat, sizeof(int64_t) * (triples + 1)), "adjacency scratch");
  XG_BUILD_CUDA(scratch.get(&at, sizeof(int64_t) * (triples + 1)), "adjacency scratch");
  XG_BUILD_CUDA(scratch.get(&bad, sizeof(unsigned long long) * 2), "adjacency scratch");
  XG_BUILD_CUDA(scratch.get(&count, sizeof(int64_t)), "adjacency scratch");
  XG_BUILD_CUDA(cudaMemsetAsync(bad, 0, sizeof(unsigned long long) * 2, s), "adjacency scratch");
  XG_BUILD_CUDA(cudaMemsetAsync(repeat + triples, 0, sizeof(int64_t), s), "adjacency scratch");
  if (triples > 0)
    check_kernel<<<grid_for(triples), kThreads, 0, s>>>(subjects, relations, objects, triples, row_offsets, entities,
                                                         writable, relation_count, repeat, bad);
  XG_BUILD_CUDA(cudaGetLastError(), "adjacency check kernel");
  // at[i] = edges before triple i; at[triples] = all edges before deduplication
  size_t temp_bytes = 0;
  XG_BUILD_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, temp_bytes, repeat, at, triples + 1, s), "adjacency scan");
  void* temp = nullptr;
  XG_BUILD_CUDA(scratch.get(&temp, temp_bytes), "adjacency scratch");
  XG_BUILD_CUDA(cub::DeviceScan::ExclusiveSum(temp, temp_bytes, repeat, at, triples + 1, s), "adjacency scan");
  unsigned long long bad_host[2] = {0, 0};
  int64_t expanded = 0;
  XG_BUILD_CUDA(cudaMemcpyAsync(bad_host, bad, sizeof(bad_host), cudaMemcpyDeviceToHost, s), "adjacency count");
  XG_BUILD_CUDA(cudaMemcpyAsync(&expanded, at + triples, sizeof(int64_t), cudaMemcpyDeviceToHost, s),
                "adjacency count");
  XG_BUILD_CUDA(cudaStreamSynchronize(s), "adjacency count");
  if (bad_host[0]) return build_fail(XG_EINVAL, "a triple names an entity or relation position out of range");
  *unwritable = static_cast<int64_t>(bad_host[1]);
  if (!offsets) {  // a sizing call: the capacity the edge arrays need
    *edges = expanded;
    return XG_OK;
  }
  if (capacity < expanded) return build_fail(XG_EINVAL, "edge capacity below the expanded edge count");
  if (expanded > 0 && (!edge_relations || !edge_objects)) return build_fail(XG_EINVAL, "null edge arrays");
  if (expanded == 0) {  // no writable triple: every subject's range is empty
    XG_BUILD_CUDA(cudaMemsetAsync(offsets, 0, sizeof(int64_t) * (entities + 1), s), "adjacency offsets");
    XG_BUILD_CUDA(cudaStreamSynchronize(s), "adjacency build");
    *edges = 0;
    return XG_OK;
  }
  uint64_t *keys = nullptr, *sorted = nullptr;
  unsigned long long* degree = nullptr;
  XG_BUILD_CUDA(scratch.get(&keys, sizeof(uint64_t) * expanded), "adjacency keys");
  XG_BUILD_CUDA(scratch.get(&sorted, sizeof(uint64_t) * expanded), "adjacency keys");
  XG_BUILD_CUDA(scratch.get(&degree, sizeof(unsigned long long) * (entities + 1)), "adjacency degrees");
  XG_BUILD_CUDA(cudaMemsetAsync(degree, 0, sizeof(unsigned long long) * (entities + 1), s), "adjacency degrees");
  expand_kernel<<<grid_for(triples), kThreads, 0, s>>>(subjects, relations, objects, triples, row_offsets, row_list,
                                                        repeat, at, relation_bits, row_bits, keys);
  XG_BUILD_CUDA(cudaGetLastError(), "adjacency expand kernel");
  const int end_bit = subject_bits + relation_bits + row_bits > 0 ? subject_bits + relation_bits + row_bits : 1;
  size_t sort_bytes = 0, unique_bytes = 0, scan_bytes = 0;
  XG_BUILD_CUDA(cub::DeviceRadixSort::SortKeys(nullptr, sort_bytes, keys, sorted, expanded, 0, end_bit, s),
                "adjacency sort");
  XG_BUILD_CUDA(cub::DeviceSelect::Unique(nullptr, unique_bytes, sorted, keys, count, expanded, s), "adjacency unique");
  XG_BUILD_CUDA(cub::DeviceScan::InclusiveSum(nullptr, scan_bytes, degree, offsets + 1, entities, s),
                "adjacency offsets");
  size_t need = sort_bytes > unique_bytes ? sort_bytes : unique_bytes;
  need = need > scan_bytes ? need : scan_bytes;
  void* work = nullptr;
  XG_BUILD_CUDA(scratch.get(&work, need), "adjacency scratch");
  XG_BUILD_CUDA(cub::DeviceRadixSort::SortKeys(work, sort_bytes, keys, sorted, expanded, 0, end_bit, s),
                "adjacency sort");
  XG_BUILD_CUDA(cub::DeviceSelect::Unique(work, unique_bytes, sorted, keys, count, expanded, s), "adjacency unique");
  decode_kernel<<<grid_for(expanded), kThreads, 0, s>>>(keys, count, relation_bits, row_bits, edge_relations,
                                                        edge_objects, degree);
  XG_BUILD_CUDA(cudaGetLastError(), "adjacency decode kernel");
  XG_BUILD_CUDA(cudaMemsetAsync(offsets, 0, sizeof(int64_t), s), "adjacency offsets");
  if (entities > 0)
    XG_BUILD_CUDA(cub::DeviceScan::InclusiveSum(work, scan_bytes, degree, offsets + 1, entities, s),
                  "adjacency offsets");
  XG_BUILD_CUDA(cudaMemcpyAsync(edges, count, sizeof(int64_t), cudaMemcpyDeviceToHost, s), "adjacency count");
  XG_BUILD_CUDA(cudaStreamSynchronize(s), "adjacency build");
  return XG_OK;
}

extern "C" XG_API int xg_build_label_rows(int32_t labels, const int64_t* token_off, const int32_t* token_ids,
                                          int64_t token_count, const int64_t* text_off, const uint8_t* text,
                                          int64_t text_bytes, const int32_t* owners, int32_t owner_count,
                                          int32_t vocab, const int64_t* vocab_off, const uint8_t* vocab_bytes,
                                          int64_t vocab_byte_count, const int8_t* vocab_kind, int32_t* status,
                                          int64_t* row_offsets, int32_t* row_tokens, int32_t* row_owners,
                                          int32_t* rows, int64_t* tokens, void* stream) {
  if (!rows || !tokens) return build_fail(XG_EINVAL, "null rows or tokens output");
  if (labels < 0 || token_count < 0 || text_bytes < 0 || owner_count < 0 || vocab <= 0 || vocab_byte_count < 0)
    return build_fail(XG_EINVAL, "negative size or empty vocabulary");
  if (!token_off || !text_off || !vocab_off || !vocab_kind || !status || !row_offsets ||
      (labels > 0 && (!owners || !row_owners)) || (token_count > 0 && (!token_ids || !row_tokens)) ||
      (text_bytes > 0 && !text) || (vocab_byte_count > 0 && !vocab_bytes))
    return build_fail(XG_EINVAL, "null label, text or vocabulary array");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  *rows = 0;
  *tokens = 0;
  XG_BUILD_CUDA(cudaMemsetAsync(row_offsets, 0, sizeof(int64_t), s), "label rows");
  if (labels == 0) {
    XG_BUILD_CUDA(cudaStreamSynchronize(s), "label rows");
    return XG_OK;
  }
  Scratch scratch(s);
  int32_t *selected = nullptr, *order = nullptr, *swap = nullptr, *length = nullptr, *longest = nullptr;
  uint8_t* admitted = nullptr;
  int64_t* count = nullptr;
  unsigned long long* bad = nullptr;
  uint32_t *keys = nullptr, *keys_out = nullptr;
  int64_t* lengths = nullptr;
  XG_BUILD_CUDA(scratch.get(&selected, sizeof(int32_t) * labels), "label scratch");
  XG_BUILD_CUDA(scratch.get(&order, sizeof(int32_t) * labels), "label scratch");
  XG_BUILD_CUDA(scratch.get(&swap, sizeof(int32_t) * labels), "label scratch");
  XG_BUILD_CUDA(scratch.get(&length, sizeof(int32_t) * labels), "label scratch");
  XG_BUILD_CUDA(scratch.get(&admitted, labels), "label scratch");
  XG_BUILD_CUDA(scratch.get(&count, 3 * sizeof(int64_t)), "label scratch");  // count, longest, bad: 8 bytes each
  longest = reinterpret_cast<int32_t*>(count + 1);
  bad = reinterpret_cast<unsigned long long*>(count + 2);
  XG_BUILD_CUDA(scratch.get(&keys, sizeof(uint32_t) * labels), "label scratch");
  XG_BUILD_CUDA(scratch.get(&keys_out, sizeof(uint32_t) * labels), "label scratch");
  XG_BUILD_CUDA(scratch.get(&lengths, sizeof(int64_t) * labels), "label scratch");
  XG_BUILD_CUDA(cudaMemsetAsync(bad, 0, sizeof(unsigned long long), s), "label scratch");
  admit_labels_kernel<<<grid_for(static_cast<int64_t>(labels) * 32), kThreads, 0, s>>>(
      labels, token_off, token_ids, token_count, text_off, text, text_bytes, owners, owner_count, vocab, vocab_off,
      vocab_bytes, vocab_byte_count, vocab_kind, status, selected, admitted, length, bad);
  XG_BUILD_CUDA(cudaGetLastError(), "label admission kernel");
  const int32_t token_bits = bits_for(static_cast<int64_t>(vocab) + 1), owner_bits = bits_for(owner_count);
  size_t select_bytes = 0, max_bytes = 0, sort_bytes = 0, scan_bytes = 0;
  XG_BUILD_CUDA(cub::DeviceSelect::Flagged(nullptr, select_bytes, selected, admitted, order, count, labels, s),
                "label select");
  XG_BUILD_CUDA(cub::DeviceReduce::Max(nullptr, max_bytes, length, longest, labels, s), "label lengths");
  XG_BUILD_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, keys, keys_out, order, swap, labels, 0,
                                                token_bits > owner_bits ? token_bits : owner_bits, s),
                "label sort");
  XG_BUILD_CUDA(cub::DeviceScan::InclusiveSum(nullptr, scan_bytes, lengths, row_offsets + 1, labels, s),
                "label offsets");
  size_t need = select_bytes > max_bytes ? select_bytes : max_bytes;
  need = need > sort_bytes ? need : sort_bytes;
  need = need > scan_bytes ? need : scan_bytes;
  void* work = nullptr;
  XG_BUILD_CUDA(scratch.get(&work, need), "label scratch");
  XG_BUILD_CUDA(cub::DeviceSelect::Flagged(work, select_bytes, selected, admitted, order, count, labels, s),
                "label select");
  XG_BUILD_CUDA(cub::DeviceReduce::Max(work, max_bytes, length, longest, labels, s), "label lengths");
  int64_t admitted_rows = 0;
  int32_t depth_count = 0;
  unsigned long long bad_host = 0;
  XG_BUILD_CUDA(cudaMemcpyAsync(&admitted_rows, count, sizeof(int64_t), cudaMemcpyDeviceToHost, s), "label count");
  XG_BUILD_CUDA(cudaMemcpyAsync(&depth_count, longest, sizeof(int32_t), cudaMemcpyDeviceToHost, s), "label count");
  XG_BUILD_CUDA(cudaMemcpyAsync(&bad_host, bad, sizeof(bad_host), cudaMemcpyDeviceToHost, s), "label count");
  XG_BUILD_CUDA(cudaStreamSynchronize(s), "label count");
  if (bad_host) return build_fail(XG_EINVAL, "label or vocabulary offsets outside their arrays, or an owner out of range");
  if (admitted_rows == 0) {
    XG_BUILD_CUDA(cudaStreamSynchronize(s), "label rows");
    return XG_OK;
  }
  const int n = static_cast<int>(admitted_rows);
  // LSD: the owner first (least significant), then depths from the deepest to the first
  for (int32_t depth = -1; depth < depth_count; ++depth) {
    const int32_t d = depth < 0 ? -1 : depth_count - 1 - depth;
    label_keys_kernel<<<grid_for(n), kThreads, 0, s>>>(order, count, token_off, token_ids, owners, d, keys);
    XG_BUILD_CUDA(cudaGetLastError(), "label key kernel");
    XG_BUILD_CUDA(cub::DeviceRadixSort::SortPairs(work, sort_bytes, keys, keys_out, order, swap, n, 0,
                                                  d < 0 ? (owner_bits > 0 ? owner_bits : 1) : token_bits, s),
                  "label sort");
    int32_t* t = order;
    order = swap;
    swap = t;
  }
  row_lengths_kernel<<<grid_for(n), kThreads, 0, s>>>(order, count, token_off, owners, lengths, row_owners);
  XG_BUILD_CUDA(cudaGetLastError(), "label length kernel");
  XG_BUILD_CUDA(cub::DeviceScan::InclusiveSum(work, scan_bytes, lengths, row_offsets + 1, n, s), "label offsets");
  row_tokens_kernel<<<grid_for(static_cast<int64_t>(n) * 32), kThreads, 0, s>>>(order, count, token_off, token_ids,
                                                                              row_offsets, row_tokens);
  XG_BUILD_CUDA(cudaGetLastError(), "label token kernel");
  int64_t total = 0;
  XG_BUILD_CUDA(cudaMemcpyAsync(&total, row_offsets + n, sizeof(int64_t), cudaMemcpyDeviceToHost, s), "label count");
  XG_BUILD_CUDA(cudaStreamSynchronize(s), "label rows");
  *rows = n;
  *tokens = total;
  return XG_OK;
}
