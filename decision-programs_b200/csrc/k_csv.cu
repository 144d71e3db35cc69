// CSV input transport on the GPU (see csv.h).
//
// Structure (the reference's read(), native/decision_programs_csv.hpp:11-24):
//  * the text is cut into 4 KB blocks; the quote count of every block and its
//    exclusive scan give each byte's quote parity, so a ',' / '\r' / '\n' is
//    structural exactly when the parity before it is even ('\n' right after a
//    structural '\r' belongs to it); structural delimiters are numbered by a
//    second count and scan, and written in order with their kind;
//  * one thread per field checks the quoting rules (a quoted field opens at
//    its first byte, "" is an escaped quote, only blanks may follow the
//    closing quote; a quote anywhere in an unquoted field is an error) and
//    keeps the smallest offending byte offset: read() stops at the first
//    offending byte, so the smallest offset carries its message.  An odd total
//    of quotes with no earlier error is an unterminated quoted field;
//  * records are numbered by a scan over the record ends; a record that is a
//    single empty field is dropped, and every other record must have the
//    first record's field count.
// Decoding (decode(), :36-67): the first record is read back for the target
// and header decisions (a handful of strings), then one thread per data cell
// parses it (dec2f.cuh: the reference's feature() and class-label rules,
// correctly rounded) into the row-major fp32 matrix.  Errors keep the
// reference's order (record, then column, the target after the features) by
// taking the smallest (record, column) key.  Non-numeric class labels are
// numbered in order of first appearance through a device hash table (64-bit
// FNV-1a of the trimmed label, every row's label compared byte for byte with
// its slot's first holder, so a hash collision fails the call instead of
// merging labels).
#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <vector>

#include "csv.h"
#include "dec2f.cuh"
#include "json.h"

namespace dp {

namespace {

constexpr int kCsvThreads = 256;
constexpr int kBytesPerThread = 16;
constexpr u64 kBlockBytes = u64(kCsvThreads) * kBytesPerThread;  // 4096
constexpr u32 kNoRow32 = 0xffffffffu;

// error kinds, in the low byte of an error key (key = position << 8 | kind)
enum : u32 {
  kErrAfterClose = 1,     // "CSV characters after closing quote"
  kErrQuoteInside = 2,    // "CSV quote inside unquoted field"
  kErrFeature = 3,        // "invalid finite-FP32 CSV feature at record R, column C"
  kErrEmptyTarget = 4,    // "empty CSV target at record R"
  kErrTargetMax = 5,      // "CSV target exceeds supported class ID"
};
// field flags
enum : u32 { kQuoted = 1, kEscape = 2, kContentEmpty = 4 };

__device__ __forceinline__ u64 block_scan_u64(u64 v, u64* total) {
  __shared__ u64 warp_sums[kCsvThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  u64 x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const u64 y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    u64 w = lane < kCsvThreads / 32 ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const u64 y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kCsvThreads / 32) warp_sums[lane] = w;
  }
  __syncthreads();
  const u64 before = (warp ? warp_sums[warp - 1] : 0) + x - v;
  if (total) *total = warp_sums[kCsvThreads / 32 - 1];
  __syncthreads();
  return before;
}

// ---- generic exclusive scan of u64 values
__global__ void k_scan_block_sums(const u64* __restrict__ in, u64 n, u64* __restrict__ sums) {
  const u64 base = u64(blockIdx.x) * kCsvThreads * 4;
  u64 v = 0;
  for (int k = 0; k < 4; ++k) {
    const u64 i = base + u64(threadIdx.x) * 4 + k;
    if (i < n) v += in[i];
  }
  u64 total = 0;
  block_scan_u64(v, &total);
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}
__global__ void k_scan_sums(u64* sums, u64 nb, u64* total_out) {
  u64 carry = 0;
  for (u64 c = 0; c < nb; c += kCsvThreads) {
    const u64 i = c + threadIdx.x;
    const u64 v = i < nb ? sums[i] : 0;
    u64 tot = 0;
    const u64 ex = block_scan_u64(v, &tot);
    if (i < nb) sums[i] = carry + ex;
    carry += tot;
  }
  if (threadIdx.x == 0 && total_out) *total_out = carry;
}
__global__ void k_scan_apply(const u64* __restrict__ in, u64 n, const u64* __restrict__ sums, u64* __restrict__ out) {
  const u64 base = u64(blockIdx.x) * kCsvThreads * 4;
  u64 v[4], s = 0;
  for (int k = 0; k < 4; ++k) {
    const u64 i = base + u64(threadIdx.x) * 4 + k;
    v[k] = i < n ? in[i] : 0;
    s += v[k];
  }
  u64 ex = block_scan_u64(s, nullptr) + sums[blockIdx.x];
  for (int k = 0; k < 4; ++k) {
    const u64 i = base + u64(threadIdx.x) * 4 + k;
    if (i < n) out[i] = ex;
    ex += v[k];
  }
}
// out[i] = sum in[0, i); *total = the whole sum (device).  `tmp` is scratch.
void exclusive_scan(const u64* in, u64* out, u64 n, u64* total, DevBuf<u64>& tmp, cudaStream_t s) {
  const u64 per = u64(kCsvThreads) * 4;
  const u64 nb = std::max<u64>(1, (n + per - 1) / per);
  tmp.reserve(nb);
  if (n) k_scan_block_sums<<<u32(nb), kCsvThreads, 0, s>>>(in, n, tmp.get());
  else DP_CUDA(cudaMemsetAsync(tmp.get(), 0, sizeof(u64), s));
  k_scan_sums<<<1, kCsvThreads, 0, s>>>(tmp.get(), nb, total);
  if (n) k_scan_apply<<<u32(nb), kCsvThreads, 0, s>>>(in, n, tmp.get(), out);
  after_launch("csv scan");
}

// ---- structure
__global__ void k_quote_counts(const u8* __restrict__ text, u64 n, u64* __restrict__ counts) {
  const u64 base = u64(blockIdx.x) * kBlockBytes + u64(threadIdx.x) * kBytesPerThread;
  u64 q = 0;
  for (int k = 0; k < kBytesPerThread; ++k) q += (base + k < n && text[base + k] == '"');
  u64 total = 0;
  block_scan_u64(q, &total);
  if (threadIdx.x == 0) counts[blockIdx.x] = total;
}

// Structural delimiters of this thread's bytes.  The count pass stores the
// block's delimiter and record-end counts; the write pass stores every
// delimiter's position in order and, for each record end, that delimiter's
// index (so record r starts at field rec_end[r - 1] + 1).
template <bool WRITE>
__device__ __forceinline__ void delimiters(const u8* __restrict__ text, u64 n, const u64* __restrict__ qbase,
                                           const u64* __restrict__ dbase, const u64* __restrict__ rbase,
                                           u64* __restrict__ pos, u64* __restrict__ rec_end, u64* __restrict__ counts,
                                           u64* __restrict__ rcounts) {
  const u64 base = u64(blockIdx.x) * kBlockBytes + u64(threadIdx.x) * kBytesPerThread;
  u64 q = 0;
  for (int k = 0; k < kBytesPerThread; ++k) q += (base + k < n && text[base + k] == '"');
  const u64 qbefore = qbase[blockIdx.x] + block_scan_u64(q, nullptr);
  u32 parity = u32(qbefore & 1u);
  u64 d = 0, r = 0;
  const u8 prev0 = base > 0 && base - 1 < n ? text[base - 1] : u8(0);
  u8 prev = prev0;
  for (int k = 0; k < kBytesPerThread; ++k) {
    const u64 i = base + k;
    if (i >= n) break;
    const u8 c = text[i];
    if (c == '"') {
      parity ^= 1u;
    } else if (!parity && (c == ',' || c == '\r' || (c == '\n' && prev != '\r'))) {
      ++d;
      r += c != ',';
    }
    prev = c;
  }
  if (!WRITE) {
    u64 dt = 0, rt = 0;
    block_scan_u64(d, &dt);
    block_scan_u64(r, &rt);
    if (threadIdx.x == 0) {
      counts[blockIdx.x] = dt;
      rcounts[blockIdx.x] = rt;
    }
    return;
  }
  u64 at = dbase[blockIdx.x] + block_scan_u64(d, nullptr);
  u64 rat = rbase[blockIdx.x] + block_scan_u64(r, nullptr);
  parity = u32(qbefore & 1u);
  prev = prev0;
  for (int k = 0; k < kBytesPerThread; ++k) {
    const u64 i = base + k;
    if (i >= n) break;
    const u8 c = text[i];
    if (c == '"') {
      parity ^= 1u;
    } else if (!parity && (c == ',' || c == '\r' || (c == '\n' && prev != '\r'))) {
      pos[at] = i;
      if (c != ',') rec_end[rat++] = at;
      ++at;
    }
    prev = c;
  }
}
__global__ void k_delim_counts(const u8* __restrict__ text, u64 n, const u64* __restrict__ qbase,
                               u64* __restrict__ counts, u64* __restrict__ rcounts) {
  delimiters<false>(text, n, qbase, nullptr, nullptr, nullptr, nullptr, counts, rcounts);
}
__global__ void k_delim_write(const u8* __restrict__ text, u64 n, const u64* __restrict__ qbase,
                              const u64* __restrict__ dbase, const u64* __restrict__ rbase, u64* __restrict__ pos,
                              u64* __restrict__ rec_end) {
  delimiters<true>(text, n, qbase, dbase, rbase, pos, rec_end, nullptr, nullptr);
}

// byte range of field j: after the previous delimiter (and the '\n' of a
// "\r\n"), up to its own delimiter or the end of the text
__device__ __forceinline__ void field_range(const u8* text, u64 n, const u64* dpos, u64 ndelim, u64 j, u64* s,
                                            u64* e) {
  u64 b = 0;
  if (j > 0) {
    b = dpos[j - 1] + 1;
    if (text[dpos[j - 1]] == '\r' && b < n && text[b] == '\n') ++b;
  }
  *s = b;
  *e = j < ndelim ? dpos[j] : n;
}

__global__ void k_fields(const u8* __restrict__ text, u64 n, const u64* __restrict__ dpos, u64 ndelim, u64 nf,
                         u32* __restrict__ clen, u8* __restrict__ flags,
                         unsigned long long* __restrict__ err) {
  const u64 j = u64(blockIdx.x) * blockDim.x + threadIdx.x;
  if (j >= nf) return;
  u64 s, e;
  field_range(text, n, dpos, ndelim, j, &s, &e);
  u32 fl = 0;
  u64 cs = s, ce = e;
  if (e > s && text[s] == '"') {
    fl |= kQuoted;
    u64 i = s + 1, close = e;
    while (i < e) {
      if (text[i] == '"') {
        if (i + 1 < e && text[i + 1] == '"') {
          fl |= kEscape;
          i += 2;
          continue;
        }
        close = i;
        break;
      }
      ++i;
    }
    cs = s + 1;
    ce = close;  // = e when the quote never closes (the text ends inside it)
    for (u64 k = close + 1; k < e; ++k) {
      const u8 c = text[k];
      if (c != ' ' && c != '\t') {
        atomicMin(err, (static_cast<unsigned long long>(k) << 8) | kErrAfterClose);
        break;
      }
    }
  } else {
    for (u64 k = s; k < e; ++k)
      if (text[k] == '"') {
        atomicMin(err, (static_cast<unsigned long long>(k) << 8) | kErrQuoteInside);
        break;
      }
  }
  if (ce == cs) fl |= kContentEmpty;
  clen[j] = u32(ce - cs < 0xffffffffull ? ce - cs : 0xffffffffull);
  flags[j] = u8(fl);
}

// record r's first field: 0, or the field after record end r - 1
__global__ void k_rec_first(const u64* __restrict__ rec_end, u64 nrec, u64 nf, u64* __restrict__ rec_first) {
  const u64 r = u64(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r > nrec) return;
  rec_first[r] = r == 0 ? 0 : (r == nrec ? nf : rec_end[r - 1] + 1);
}
__global__ void k_records(const u64* __restrict__ rec_first, u64 nrec, const u8* __restrict__ flags,
                          u64* __restrict__ kept, unsigned long long* __restrict__ cmin,
                          unsigned long long* __restrict__ cmax) {
  const u64 r = u64(blockIdx.x) * blockDim.x + threadIdx.x;
  unsigned long long lo = ~0ull, hi = 0;
  if (r < nrec) {
    const u64 cnt = rec_first[r + 1] - rec_first[r];
    const bool drop = cnt == 1 && (flags[rec_first[r]] & kContentEmpty);
    kept[r] = drop ? 0 : 1;
    if (!drop) lo = hi = cnt;
  }
  // one pair of atomics per warp
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if ((threadIdx.x & 31) == 0 && hi) {
    atomicMin(cmin, lo);
    atomicMax(cmax, hi);
  }
}
__global__ void k_compact(const u64* __restrict__ kept, const u64* __restrict__ kidx, u64 nrec, u64* __restrict__ list) {
  const u64 r = u64(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r < nrec && kept[r]) list[kidx[r]] = r;
}

// ---- decoding
struct Cells {
  const u8* text;
  u64 n;
  const u64* dpos;
  u64 ndelim;
  const u8* flags;
  const u32* clen;
  const u64* rec_first;
  const u64* kept_list;
  u64 first;    // 1 with a header record
  u64 rows;
  u32 columns;
  u32 target;   // == columns when there is none
  u32 features;
};

__device__ __forceinline__ u64 cell_field(const Cells& c, u64 row, u32 col) {
  return c.rec_first[c.kept_list[c.first + row]] + col;
}
// first content byte of field j (after the opening quote of a quoted field)
__device__ __forceinline__ const u8* content(const Cells& c, u64 j) {
  u64 s, e;
  field_range(c.text, c.n, c.dpos, c.ndelim, j, &s, &e);
  return c.text + s + ((c.flags[j] & kQuoted) ? 1 : 0);
}

__global__ void k_labels_numeric(Cells c, u32* __restrict__ numeric) {
  const u64 row = u64(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= c.rows) return;
  const u64 j = cell_field(c, row, c.target);
  u32 v;
  if (!dec::parse_label_token(content(c, j), c.clen[j], &v)) atomicAnd(numeric, 0u);
}

__global__ void k_cells(Cells c, bool numeric, float* __restrict__ values, u32* __restrict__ labels,
                        unsigned long long* __restrict__ err, u32* __restrict__ max_label) {
  const u64 t = u64(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= c.rows * c.columns) return;
  const u64 row = t / c.columns;
  const u32 col = u32(t % c.columns);
  const u64 j = cell_field(c, row, col);
  const u8* p = content(c, j);
  const u32 len = c.clen[j];
  const unsigned long long rec = c.first + row;
  if (col == c.target) {
    if (numeric) {
      u32 v = 0;
      dec::parse_label_token(p, len, &v);  // every label parsed in the check pass
      if (v == 0xffffffffu) {
        atomicMin(err, ((rec * (c.columns + 1ull) + c.columns) << 8) | kErrTargetMax);
        return;
      }
      labels[row] = v;
      atomicMax(max_label, v);
    } else {
      u32 b = 0, e = len;
      while (b < e && dec::is_space(p[b])) ++b;
      while (e > b && dec::is_space(p[e - 1])) --e;
      if (b == e) atomicMin(err, ((rec * (c.columns + 1ull) + c.columns) << 8) | kErrEmptyTarget);
    }
    return;
  }
  float v;
  if (!dec::parse_feature_token(p, len, &v)) {
    atomicMin(err, ((rec * (c.columns + 1ull) + col) << 8) | kErrFeature);
    return;
  }
  const u32 fc = col < c.target ? col : col - 1;
  values[row * c.features + fc] = v;
}

// trimmed label [b, e) of a quoted-or-not content; `esc` when "" pairs occur
__device__ __forceinline__ void label_span(const u8* p, u32 len, u32* b, u32* e) {
  u32 x = 0, y = len;
  while (x < y && dec::is_space(p[x])) ++x;
  while (y > x && dec::is_space(p[y - 1])) --y;
  *b = x;
  *e = y;
}
// next byte of the unescaped content at *i (a "" pair reads as one quote)
__device__ __forceinline__ u8 next_byte(const u8* p, u32* i, bool esc) {
  const u8 c = p[*i];
  *i += (esc && c == '"') ? 2 : 1;
  return c;
}

struct LabelTable {
  unsigned long long* keys;
  u32* first_row;
  u32* dindex;
  u64 size;  // power of two
};

__global__ void k_label_insert(Cells c, const u8* __restrict__ flags, LabelTable tab, u32* __restrict__ slot_of,
                               u32* __restrict__ overflow) {
  const u64 row = u64(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= c.rows) return;
  const u64 j = cell_field(c, row, c.target);
  const u8* p = content(c, j);
  const bool esc = flags[j] & kEscape;
  u32 b, e;
  label_span(p, c.clen[j], &b, &e);
  unsigned long long h = 1469598103934665603ull;  // FNV-1a, 64-bit
  for (u32 i = b; i < e;) {
    h ^= next_byte(p, &i, esc);
    h *= 1099511628211ull;
  }
  const unsigned long long key = h | 1ull;
  u64 slot = key & (tab.size - 1);
  for (u64 probe = 0;; ++probe) {
    if (probe >= tab.size) {
      atomicOr(overflow, 1u);
      slot_of[row] = kNoRow32;
      return;
    }
    const unsigned long long old = atomicCAS(tab.keys + slot, 0ull, key);
    if (old == 0ull || old == key) break;
    slot = (slot + 1) & (tab.size - 1);
  }
  atomicMin(tab.first_row + slot, u32(row));
  slot_of[row] = u32(slot);
}

// every row's label equals the first holder's of its slot, byte for byte
__global__ void k_label_verify(Cells c, const u8* __restrict__ flags, LabelTable tab, const u32* __restrict__ slot_of,
                               u32* __restrict__ collision) {
  const u64 row = u64(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= c.rows || slot_of[row] == kNoRow32) return;
  const u64 rep = tab.first_row[slot_of[row]];
  if (rep == row) return;
  const u64 j = cell_field(c, row, c.target), k = cell_field(c, rep, c.target);
  const u8* p = content(c, j);
  const u8* q = content(c, k);
  const bool pe = flags[j] & kEscape, qe = flags[k] & kEscape;
  u32 pb, pend, qb, qend;
  label_span(p, c.clen[j], &pb, &pend);
  label_span(q, c.clen[k], &qb, &qend);
  u32 i = pb, m = qb;
  while (i < pend && m < qend)
    if (next_byte(p, &i, pe) != next_byte(q, &m, qe)) {
      atomicOr(collision, 1u);
      return;
    }
  if (i < pend || m < qend) atomicOr(collision, 1u);
}

__global__ void k_label_distinct(LabelTable tab, u32* __restrict__ ndist, u32* __restrict__ dist_first) {
  const u64 s = u64(blockIdx.x) * blockDim.x + threadIdx.x;
  if (s >= tab.size || tab.keys[s] == 0ull) return;
  const u32 d = atomicAdd(ndist, 1u);
  tab.dindex[s] = d;
  dist_first[d] = tab.first_row[s];
}

// unescaped, trimmed label of each distinct class into one buffer
__global__ void k_label_lengths(Cells c, const u8* __restrict__ flags, const u32* __restrict__ dist_first, u32 nd,
                                u64* __restrict__ lens) {
  const u32 d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= nd) return;
  const u64 j = cell_field(c, dist_first[d], c.target);
  const u8* p = content(c, j);
  const bool esc = flags[j] & kEscape;
  u32 b, e;
  label_span(p, c.clen[j], &b, &e);
  u64 n = 0;
  for (u32 i = b; i < e; ++n) next_byte(p, &i, esc);
  lens[d] = n;
}
__global__ void k_label_gather(Cells c, const u8* __restrict__ flags, const u32* __restrict__ dist_first, u32 nd,
                               const u64* __restrict__ offs, u8* __restrict__ out) {
  const u32 d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= nd) return;
  const u64 j = cell_field(c, dist_first[d], c.target);
  const u8* p = content(c, j);
  const bool esc = flags[j] & kEscape;
  u32 b, e;
  label_span(p, c.clen[j], &b, &e);
  u64 o = offs[d];
  for (u32 i = b; i < e;) out[o++] = next_byte(p, &i, esc);
}
__global__ void k_label_assign(u64 rows, const u32* __restrict__ slot_of, const u32* __restrict__ dindex,
                               const u32* __restrict__ id_of, u32* __restrict__ labels) {
  const u64 row = u64(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row < rows) labels[row] = id_of[dindex[slot_of[row]]];
}

u32 grid_for(u64 n, u32 threads = 256) {
  const u64 g = (n + threads - 1) / threads;
  need(g < (u64(1) << 31), "CSV input too large for one launch");
  return u32(std::max<u64>(g, 1));
}

template <class T>
T read1(const T* d, cudaStream_t s) {
  T v;
  DP_CUDA(cudaMemcpyAsync(&v, d, sizeof(T), cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaStreamSynchronize(s));
  return v;
}

[[noreturn]] void bad(const std::string& m) { throw std::invalid_argument(m); }

bool host_feature(const std::string& t) {
  float v;
  return dec::parse_feature_token(reinterpret_cast<const unsigned char*>(t.data()), u32(t.size()), &v);
}

}  // namespace

bool csv_parse_feature_host(const unsigned char* p, u32 n, float* value) {
  return dec::parse_feature_token(p, n, value);
}

std::unique_ptr<CsvDense> csv_decode(const char* bytes, u64 n, const std::string& target,
                                     const std::string& header_mode, cudaStream_t s) {
  NvtxRange nv("dp_gbdt: CSV decode");
  auto out = std::make_unique<CsvDense>();
  // device time of the decode: [ev0, evA) before the second allocation and
  // [evB, ev1) after it (the allocation itself is host time)
  cudaEvent_t ev0, evA, evB, ev1;
  DP_CUDA(cudaEventCreate(&ev0));
  DP_CUDA(cudaEventCreate(&evA));
  DP_CUDA(cudaEventCreate(&evB));
  DP_CUDA(cudaEventCreate(&ev1));
  struct Events {
    cudaEvent_t e[4];
    ~Events() {
      for (auto x : e) cudaEventDestroy(x);
    }
  } events{{ev0, evA, evB, ev1}};
  // device memory in two slabs (a cudaMalloc / cudaFree costs about half a
  // millisecond each on this GPU): what the structure pass needs, then the
  // per-delimiter, per-field and per-record arrays once their count is known
  std::vector<DevBuf<u8>> slabs;
  const u64 nb = std::max<u64>(1, (n + kBlockBytes - 1) / kBlockBytes);
  need(nb < (u64(1) << 31), "CSV input too large");
  DevBuf<u8> text;
  DevBuf<unsigned long long> sc;
  DevBuf<u64> qcnt, qbase, dcnt, dbase, rcnt, rbase, tmp;
  {
    SlabPlan plan;
    plan.want(text, nb * kBlockBytes);  // zero-padded to whole blocks
    plan.want(sc, 8);
    plan.want(qcnt, nb);
    plan.want(qbase, nb);
    plan.want(dcnt, nb);
    plan.want(dbase, nb);
    plan.want(rcnt, nb);
    plan.want(rbase, nb);
    plan.want(tmp, nb / (kCsvThreads * 4) + 2);
    plan.commit(slabs);
  }
  if (n) DP_CUDA(cudaMemcpyAsync(text.get(), bytes, n, cudaMemcpyHostToDevice, s));
  DP_CUDA(cudaMemsetAsync(text.get() + n, 0, nb * kBlockBytes - n, s));
  DP_CUDA(cudaEventRecord(ev0, s));

  // small device scalars: [0] quote total, [1] delimiter total, [2] error key,
  // [3] min count, [4] max count, [5] kept total, [6] record-end total
  const unsigned long long init[8] = {0, 0, ~0ull, ~0ull, 0, 0, 0, 0};
  DP_CUDA(cudaMemcpyAsync(sc.get(), init, sizeof init, cudaMemcpyHostToDevice, s));
  u64* sq = reinterpret_cast<u64*>(sc.get());

  // quote parity and structural delimiters
  k_quote_counts<<<u32(nb), kCsvThreads, 0, s>>>(text.get(), n, qcnt.get());
  exclusive_scan(qcnt.get(), qbase.get(), nb, sq + 0, tmp, s);
  k_delim_counts<<<u32(nb), kCsvThreads, 0, s>>>(text.get(), n, qbase.get(), dcnt.get(), rcnt.get());
  exclusive_scan(dcnt.get(), dbase.get(), nb, sq + 1, tmp, s);
  exclusive_scan(rcnt.get(), rbase.get(), nb, sq + 6, tmp, s);
  after_launch("csv delimiters");
  u64 totals[7];
  DP_CUDA(cudaMemcpyAsync(totals, sq, sizeof totals, cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaStreamSynchronize(s));
  const u64 ndelim = totals[1], nends = totals[6];
  DP_CUDA(cudaEventRecord(evA, s));
  // fields: one per delimiter plus possibly a trailing one; records likewise
  const u64 nfmax = ndelim + 1, nrecmax = nends + 1;
  DevBuf<u64> dpos, rec_end, rec_first, kept, kidx, kept_list, tmp2;
  DevBuf<u8> flags;
  DevBuf<u32> clen, aux;
  {
    SlabPlan plan;
    plan.want(dpos, nfmax);
    plan.want(rec_end, nrecmax);
    plan.want(clen, nfmax);
    plan.want(flags, nfmax);
    plan.want(rec_first, nrecmax + 1);
    plan.want(kept, nrecmax);
    plan.want(kidx, nrecmax);
    plan.want(kept_list, nrecmax);
    plan.want(tmp2, nrecmax / (kCsvThreads * 4) + 2);
    plan.want(aux, 4);
    plan.commit(slabs);
  }
  DP_CUDA(cudaEventRecord(evB, s));
  k_delim_write<<<u32(nb), kCsvThreads, 0, s>>>(text.get(), n, qbase.get(), dbase.get(), rbase.get(), dpos.get(),
                                                rec_end.get());
  after_launch("csv delimiters");

  // the trailing field counts when it has bytes or follows a ','
  u64 last_pos = 0;
  if (ndelim) {
    DP_CUDA(cudaMemcpyAsync(&last_pos, dpos.get() + ndelim - 1, sizeof(u64), cudaMemcpyDeviceToHost, s));
    DP_CUDA(cudaStreamSynchronize(s));
  }
  u64 tail_start = 0;
  if (ndelim) {
    tail_start = last_pos + 1;
    if (bytes[last_pos] == '\r' && tail_start < n && bytes[tail_start] == '\n') ++tail_start;
  }
  const bool tail = tail_start < n || (ndelim && bytes[last_pos] == ',');
  const u64 nf = ndelim + (tail ? 1 : 0);

  if (nf)
    k_fields<<<grid_for(nf), 256, 0, s>>>(text.get(), n, dpos.get(), ndelim, nf, clen.get(),
                                          flags.get(), sc.get() + 2);
  after_launch("csv fields");
  const unsigned long long qerr = read1(sc.get() + 2, s);
  const u64 quotes = totals[0];
  if (qerr != ~0ull) bad((qerr & 0xff) == kErrAfterClose ? "CSV characters after closing quote"
                                                          : "CSV quote inside unquoted field");
  if (quotes & 1u) bad("CSV unterminated quoted field");

  // records
  const u64 nrec = nends + (tail ? 1 : 0);
  if (nrec == 0) bad("CSV contains no records");
  k_rec_first<<<grid_for(nrec + 1), 256, 0, s>>>(rec_end.get(), nrec, nf, rec_first.get());
  k_records<<<grid_for(nrec), 256, 0, s>>>(rec_first.get(), nrec, flags.get(), kept.get(), sc.get() + 3, sc.get() + 4);
  exclusive_scan(kept.get(), kidx.get(), nrec, sq + 5, tmp2, s);
  k_compact<<<grid_for(nrec), 256, 0, s>>>(kept.get(), kidx.get(), nrec, kept_list.get());
  after_launch("csv records");
  unsigned long long h[8];
  DP_CUDA(cudaMemcpyAsync(h, sc.get(), sizeof h, cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaStreamSynchronize(s));
  const u64 nkept = h[5];
  if (nkept == 0) bad("CSV contains no records");
  if (h[3] != h[4]) bad("CSV rows have different column counts");
  const u64 columns = h[3];

  // the first record, on the host (target and header decisions)
  u64 r0 = 0, f0 = 0;
  DP_CUDA(cudaMemcpyAsync(&r0, kept_list.get(), sizeof(u64), cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaStreamSynchronize(s));
  DP_CUDA(cudaMemcpyAsync(&f0, rec_first.get() + r0, sizeof(u64), cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaStreamSynchronize(s));
  std::vector<u64> h_cs(columns);
  std::vector<u32> h_cl(columns);
  std::vector<u8> h_fl(columns);
  // content starts from the delimiter positions: field j starts after
  // delimiter j - 1 (and the '\n' of a "\r\n"), plus an opening quote
  std::vector<u64> h_dp(columns + 1, 0);
  if (f0 > 0)
    DP_CUDA(cudaMemcpyAsync(h_dp.data(), dpos.get() + f0 - 1, std::min<u64>(columns, ndelim - (f0 - 1)) * sizeof(u64),
                            cudaMemcpyDeviceToHost, s));
  else if (ndelim)
    DP_CUDA(cudaMemcpyAsync(h_dp.data() + 1, dpos.get(), std::min<u64>(columns - 1, ndelim) * sizeof(u64),
                            cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaMemcpyAsync(h_cl.data(), clen.get() + f0, columns * sizeof(u32), cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaMemcpyAsync(h_fl.data(), flags.get() + f0, columns, cudaMemcpyDeviceToHost, s));
  DP_CUDA(cudaStreamSynchronize(s));
  for (u64 c = 0; c < columns; ++c) {
    const u64 j = f0 + c;
    u64 st = 0;
    if (j > 0) {
      st = h_dp[c] + 1;  // h_dp[c] = dpos[j - 1]
      if (bytes[h_dp[c]] == '\r' && st < n && bytes[st] == '\n') ++st;
    }
    h_cs[c] = st + ((h_fl[c] & kQuoted) ? 1 : 0);
  }
  std::vector<std::string> rec0(columns);
  for (u64 c = 0; c < columns; ++c) {
    std::string v;
    for (u64 i = h_cs[c]; i < h_cs[c] + h_cl[c]; ++i) {
      v.push_back(bytes[i]);
      if ((h_fl[c] & kEscape) && bytes[i] == '"') ++i;  // "" reads as one quote
    }
    rec0[c] = std::move(v);
  }

  // decode(): target, header, shape (native/decision_programs_csv.hpp:37-48)
  u64 target_index = columns;
  bool header = false;
  if (!target.empty()) {
    auto found = std::find(rec0.begin(), rec0.end(), target);
    if (found != rec0.end()) {
      target_index = u64(found - rec0.begin());
      header = true;
    } else if (target == "last") {
      target_index = columns - 1;
    } else {
      u64 v = 0;
      bool ok = true;
      for (char ch : target) {
        if (ch < '0' || ch > '9') { ok = false; break; }
        const u64 nv = v * 10 + u64(ch - '0');
        if (nv / 10 != v) { ok = false; break; }
        v = nv;
      }
      if (!ok || v >= columns)
        bad("--target must name a CSV header or a zero-based column index (or last)");
      target_index = v;
    }
  }
  if (header_mode == "yes") {
    header = true;
  } else if (header_mode == "no") {
    if (header) bad("named --target requires a CSV header");
    header = false;
  } else if (header_mode == "auto") {
    if (!header)
      for (u64 c = 0; c < columns; ++c)
        if (c != target_index && !host_feature(rec0[c])) {
          header = true;
          break;
        }
  } else {
    bad("--header must be auto, yes or no");
  }
  const bool has_target = !target.empty();
  if (columns <= u64(has_target) || columns > 0xffffffffull) bad("CSV feature column count invalid");
  const u64 features = columns - u64(has_target);
  const u64 first = header ? 1 : 0;
  if (nkept <= first) bad("CSV contains no data rows");
  const u64 rows = nkept - first;
  if (rows > (~u64(0)) / (features * 4)) bad("CSV input extent overflow");
  json::Value names = json::Value::array();
  for (u64 c = 0; c < columns; ++c)
    if (c != target_index) names.push(json::Value::string(header ? rec0[c] : "feature_" + std::to_string(c)));

  out->rows = rows;
  out->features = u32(features);
  out->header = header;
  out->has_target = has_target;
  out->values.resize(std::max<u64>(rows * features, 1));
  Cells cells{text.get(), n, dpos.get(), ndelim, flags.get(), clen.get(), rec_first.get(), kept_list.get(), first, rows,
              u32(columns),
              u32(target_index), u32(features)};
  // aux: [0] numeric labels, [1] max label, [2] table overflow, [3] collision
  const u32 init_aux[4] = {1u, 0u, 0u, 0u};
  DP_CUDA(cudaMemcpyAsync(aux.get(), init_aux, sizeof init_aux, cudaMemcpyHostToDevice, s));
  bool numeric = has_target;
  if (has_target) {
    out->labels.resize(std::max<u64>(rows, 1));
    k_labels_numeric<<<grid_for(rows), 256, 0, s>>>(cells, aux.get());
    numeric = read1(aux.get(), s) != 0;
  }
  k_cells<<<grid_for(rows * columns), 256, 0, s>>>(cells, numeric, out->values.get(),
                                                  has_target ? out->labels.get() : nullptr, sc.get() + 2, aux.get() + 1);
  after_launch("csv cells");
  const unsigned long long cerr = read1(sc.get() + 2, s);
  if (cerr != ~0ull) {
    const u64 key = cerr >> 8;
    const u64 rec = key / (columns + 1), col = key % (columns + 1);
    switch (u32(cerr & 0xff)) {
      case kErrFeature:
        bad("invalid finite-FP32 CSV feature at record " + std::to_string(rec + 1) + ", column " + std::to_string(col));
      case kErrEmptyTarget:
        bad("empty CSV target at record " + std::to_string(rec + 1));
      default:
        bad("CSV target exceeds supported class ID");
    }
  }

  json::Value mapping = json::Value::null();
  if (has_target) {
    mapping = json::Value::array();
    if (numeric) {
      const u32 mx = read1(aux.get() + 1, s);
      out->classes = mx + 1;
    } else {
      // non-numeric labels: ids in order of first appearance
      u64 tsize = 1024;
      while (tsize < 2 * rows && tsize < (u64(1) << 24)) tsize <<= 1;
      DevBuf<unsigned long long> keys(tsize);
      DevBuf<u32> first_row(tsize), dindex(tsize), slot_of(rows), dist_first(tsize), ndist_d(1);
      DP_CUDA(cudaMemsetAsync(keys.get(), 0, tsize * sizeof(unsigned long long), s));
      DP_CUDA(cudaMemsetAsync(first_row.get(), 0xff, tsize * sizeof(u32), s));
      DP_CUDA(cudaMemsetAsync(ndist_d.get(), 0, sizeof(u32), s));
      const LabelTable tab{keys.get(), first_row.get(), dindex.get(), tsize};
      k_label_insert<<<grid_for(rows), 256, 0, s>>>(cells, flags.get(), tab, slot_of.get(), aux.get() + 2);
      k_label_verify<<<grid_for(rows), 256, 0, s>>>(cells, flags.get(), tab, slot_of.get(), aux.get() + 3);
      k_label_distinct<<<grid_for(tsize), 256, 0, s>>>(tab, ndist_d.get(), dist_first.get());
      after_launch("csv labels");
      u32 flags_h[4];
      DP_CUDA(cudaMemcpyAsync(flags_h, aux.get(), sizeof flags_h, cudaMemcpyDeviceToHost, s));
      const u32 nd = read1(ndist_d.get(), s);
      need(!flags_h[2], "CSV target has more distinct labels than the label table holds");
      need(!flags_h[3], "CSV target labels collide in the label hash; refusing to merge them");
      std::vector<u32> dfirst(nd);
      DP_CUDA(cudaMemcpyAsync(dfirst.data(), dist_first.get(), nd * sizeof(u32), cudaMemcpyDeviceToHost, s));
      DevBuf<u64> lens(std::max<u32>(nd, 1)), offs(std::max<u32>(nd, 1));
      k_label_lengths<<<grid_for(nd), 256, 0, s>>>(cells, flags.get(), dist_first.get(), nd, lens.get());
      std::vector<u64> hl(nd), ho(nd);
      DP_CUDA(cudaMemcpyAsync(hl.data(), lens.get(), nd * sizeof(u64), cudaMemcpyDeviceToHost, s));
      DP_CUDA(cudaStreamSynchronize(s));
      u64 total = 0;
      for (u32 d = 0; d < nd; ++d) {
        ho[d] = total;
        total += hl[d];
      }
      DevBuf<u8> strs(std::max<u64>(total, 1));
      DP_CUDA(cudaMemcpyAsync(offs.get(), ho.data(), nd * sizeof(u64), cudaMemcpyHostToDevice, s));
      k_label_gather<<<grid_for(nd), 256, 0, s>>>(cells, flags.get(), dist_first.get(), nd, offs.get(), strs.get());
      std::string hs(total, '\0');
      DP_CUDA(cudaMemcpyAsync(hs.data(), strs.get(), total, cudaMemcpyDeviceToHost, s));
      DP_CUDA(cudaStreamSynchronize(s));
      std::vector<u32> order(nd);
      for (u32 d = 0; d < nd; ++d) order[d] = d;
      std::sort(order.begin(), order.end(), [&](u32 a, u32 b) { return dfirst[a] < dfirst[b]; });
      std::vector<u32> id_of(std::max<u32>(nd, 1));
      for (u32 i = 0; i < nd; ++i) id_of[order[i]] = i;
      DevBuf<u32> id_d(std::max<u32>(nd, 1));
      DP_CUDA(cudaMemcpyAsync(id_d.get(), id_of.data(), id_of.size() * sizeof(u32), cudaMemcpyHostToDevice, s));
      k_label_assign<<<grid_for(rows), 256, 0, s>>>(rows, slot_of.get(), dindex.get(), id_d.get(), out->labels.get());
      after_launch("csv labels");
      // the mapping, ordered by label as std::map orders std::string keys
      std::vector<std::pair<std::string, u32>> m(nd);
      for (u32 d = 0; d < nd; ++d) m[d] = {hs.substr(ho[d], hl[d]), id_of[d]};
      std::sort(m.begin(), m.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
      for (auto& [label, id] : m) {
        json::Value e = json::Value::object();
        e.set("class", json::Value::number(double(id), std::to_string(id)));
        e.set("label", json::Value::string(label));
        mapping.push(std::move(e));
      }
      out->classes = nd;
      DP_CUDA(cudaStreamSynchronize(s));
    }
  }
  DP_CUDA(cudaEventRecord(ev1, s));
  DP_CUDA(cudaEventSynchronize(ev1));
  float ms_a = 0.f, ms_b = 0.f;
  DP_CUDA(cudaEventElapsedTime(&ms_a, ev0, evA));
  DP_CUDA(cudaEventElapsedTime(&ms_b, evB, ev1));
  out->ms_device = double(ms_a) + double(ms_b);
  json::Value meta = json::Value::object();
  meta.set("header", json::Value::boolean(header));
  meta.set("names", std::move(names));
  meta.set("label_mapping", std::move(mapping));
  out->meta = meta.dump();
  return out;
}

}  // namespace dp
