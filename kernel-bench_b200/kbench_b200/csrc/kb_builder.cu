// Static builder on the device: gene-tree topologies -> clade amalgamation -> the wave layout the
// solver consumes (rows ordered by clade size, per-wave split arrays).
//
// The reference consumes this layout from an external capture and ships no builder; the host
// generator (kbench_b200/gen.py: family_from_topologies + assemble_static) defines the result,
// and this file reproduces it exactly for batches of families:
//
//   1. clade hashes: per topology, every internal node's hash is the 64-bit wrapping sum of its
//      leaves' hashes, computed bottom-up by one thread per gene leaf that climbs while it is the
//      second child to arrive at a node (an arrival counter per node; no thread ever waits);
//   2. per family, an open-addressing hash table of clades (key: clade hash) and one of splits
//      (key: clade slot << 32 | slot of the split's smaller-hash child; the other child's hash is
//      the clade's minus that one), with observed counts;
//   3. amalgamation rounds: from a snapshot of each clade's splits (a CSR rebuilt per round), every
//      split (c | o) of a clade X and every split (h1 | h2) of c proposes (h1 | h2+o) and
//      (h2 | h1+o) when h2+o (resp. h1+o) is a clade of the summed size; proposals are inserted
//      with count 0 unless present;
//   4. log2 smoothed split frequencies log2((count + alpha) / (n_obs + alpha * n_splits)) in fp64,
//      rounded to fp32;
//   5. rows: every clade, ordered by (size, more-than-one-split, family, hash) -- leaves by
//      (family, gene index) -- with a stable LSD radix sort (8-bit digits, one warp per 4,096-key
//      tile, ranks within a digit from __match_any_sync); waves are the runs of equal size; each
//      row's splits are ordered by their smaller child hash.
//
// Every array lives in a caller-provided workspace (kb_build_workspace sizes it); tables are
// probed linearly with a bound, and a full table, a malformed topology or the reserved hash value
// set status bits instead of faulting (the caller retries with larger tables or reports).

#include <climits>

#include "kb_common.cuh"
#include "kb_solver.h"

namespace {

typedef unsigned long long u64;
constexpr u64 EMPTY = ~0ull;

enum : int {
  ST_CLADE_FULL = 1,
  ST_SPLIT_FULL = 2,
  ST_RESERVED_HASH = 4,
  ST_BAD_TOPOLOGY = 8,
  ST_MISSING = 16,
  ST_OVERFLOW = 32,
};

// splitmix64 output finaliser (Steele, Lea & Flood, "Fast splittable pseudorandom number
// generators", 2014), used to spread keys over the table.
__device__ __forceinline__ u64 mix64(u64 x) {
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x;
}

// Insert `key` into keys[0..mask] (linear probing); returns the slot, -1 when the table is full.
__device__ __forceinline__ int table_insert(u64* keys, int mask, u64 key, bool* fresh) {
  int slot = (int)(mix64(key) & (u64)mask);
  for (int p = 0; p <= mask; ++p) {
    const u64 old = atomicCAS(keys + slot, EMPTY, key);
    if (old == EMPTY || old == key) {
      *fresh = old == EMPTY;
      return slot;
    }
    slot = (slot + 1) & mask;
  }
  return -1;
}

// Slot of `key` in a table that no thread modifies during the call, or -1.
__device__ __forceinline__ int table_find(const u64* keys, int mask, u64 key) {
  int slot = (int)(mix64(key) & (u64)mask);
  for (int p = 0; p <= mask; ++p) {
    const u64 k = keys[slot];
    if (k == key) return slot;
    if (k == EMPTY) return -1;
    slot = (slot + 1) & mask;
  }
  return -1;
}

__device__ __forceinline__ long long gtid() { return (long long)blockIdx.x * blockDim.x + threadIdx.x; }
__device__ __forceinline__ long long gstride() { return (long long)gridDim.x * blockDim.x; }

// ---- workspace layout -----------------------------------------------------------------------

struct Dims {
  int F, T, G, cl, sl;
  long long NN, nodes, inst, CS, SS;
};

Dims make_dims(int F, int T, int G, int cl, int sl) {
  Dims d{F, T, G, cl, sl, 0, 0, 0, 0, 0};
  d.NN = 2LL * G - 1;
  d.nodes = (long long)F * T * d.NN;
  d.inst = (long long)F * T * (G - 1);
  d.CS = (long long)F << cl;
  d.SS = (long long)F << sl;
  return d;
}

constexpr int RX_TILE = 4096;  // keys per warp tile of the radix sort
constexpr int RX_WARPS = 8;
constexpr int SC_THREADS = 1024, SC_VALS = 8, SC_TILE = SC_THREADS * SC_VALS;

long long rx_tiles(long long n) { return (n + RX_TILE - 1) / RX_TILE; }
long long sc_tiles(long long n) { return (n + SC_TILE - 1) / SC_TILE; }

// Scratch of the device-wide scans: tile sums, the total, the status word (overflow bit).
struct ScanCtx {
  long long* sums;
  long long* total;
  int* status;
};

struct Work {
  int* status;        // [8]: [0] status bits
  u64* counters;      // [8]: [0] splits added by the amalgamation
  long long* total;   // [4] scan totals
  long long* sums;    // scan tile sums
  int* npar;          // [nodes] parent of each topology node (-1: root)
  int* narr;          // [nodes] arrivals
  int* nsz;           // [nodes] clade size
  u64* nh;            // [nodes] clade hash
  u64* ckey;          // [CS] clade tables (F x 2^cl)
  int* csize;
  int* cleaf;         // gene index of a leaf clade, -1 otherwise
  int* cnspl;         // [CS+1] splits per clade
  int* cptr;          // [CS+1] CSR offsets
  int* ccur;          // [CS+1] CSR fill cursors
  int* cnobs;         // [CS] observed count per clade
  int* crow;          // [CS] row id per clade
  u64* skey;          // [SS] split tables (F x 2^sl)
  int* scount;
  int* sL;            // global clade slot of the smaller-hash child
  int* sH;            // global clade slot of the other child
  float* slp;
  int* csr;           // [SS] split slots grouped by clade
  int* rflag;         // [CS+1] compaction flags / positions
  u64* k64[2];        // [CS] sort keys (hash or gene index)
  unsigned* g32[2];   // [CS] sort keys (size << 16 | multi << 15 | family)
  unsigned* val[2];   // [CS] clade slot
  int* hist;          // radix histograms
  int* rwave;         // [CS+1] wave-start flags -> wave index (inclusive scan - 1)
  int* rsp;           // [CS+1] splits per row -> row split offsets
  int* wstart;        // [G+2] per wave
  int* wend;
  int* wmulti;        // first row with more than one split (INT_MAX: none)
  int* wfan;          // largest split count among those rows
  size_t bytes;
  ScanCtx scan() const { return ScanCtx{sums, total, status}; }
};

Work carve(void* base, const Dims& d) {
  Work w{};
  size_t off = 0;
  char* b = static_cast<char*>(base);
  auto take = [&](size_t n) -> void* {
    off = (off + 255) & ~size_t(255);
    void* p = b ? b + off : nullptr;
    off += n;
    return p;
  };
  const long long CS1 = d.CS + 1, SS1 = d.SS + 1;
  const long long scan_max = (CS1 > SS1 ? CS1 : SS1);
  w.status = (int*)take(8 * sizeof(int));
  w.counters = (u64*)take(8 * sizeof(u64));
  w.total = (long long*)take(4 * sizeof(long long));
  w.sums = (long long*)take((sc_tiles(scan_max) + 1) * sizeof(long long));
  w.npar = (int*)take(d.nodes * sizeof(int));
  w.narr = (int*)take(d.nodes * sizeof(int));
  w.nsz = (int*)take(d.nodes * sizeof(int));
  w.nh = (u64*)take(d.nodes * sizeof(u64));
  w.ckey = (u64*)take(d.CS * sizeof(u64));
  w.csize = (int*)take(d.CS * sizeof(int));
  w.cleaf = (int*)take(d.CS * sizeof(int));
  w.cnspl = (int*)take(CS1 * sizeof(int));
  w.cptr = (int*)take(CS1 * sizeof(int));
  w.ccur = (int*)take(CS1 * sizeof(int));
  w.cnobs = (int*)take(d.CS * sizeof(int));
  w.crow = (int*)take(d.CS * sizeof(int));
  w.skey = (u64*)take(d.SS * sizeof(u64));
  w.scount = (int*)take(d.SS * sizeof(int));
  w.sL = (int*)take(d.SS * sizeof(int));
  w.sH = (int*)take(d.SS * sizeof(int));
  w.slp = (float*)take(d.SS * sizeof(float));
  w.csr = (int*)take(d.SS * sizeof(int));
  w.rflag = (int*)take(CS1 * sizeof(int));
  for (int i = 0; i < 2; ++i) {
    w.k64[i] = (u64*)take(d.CS * sizeof(u64));
    w.g32[i] = (unsigned*)take(d.CS * sizeof(unsigned));
    w.val[i] = (unsigned*)take(d.CS * sizeof(unsigned));
  }
  w.hist = (int*)take((256 * rx_tiles(d.CS) + 1) * sizeof(int));
  w.rwave = (int*)take(CS1 * sizeof(int));
  w.rsp = (int*)take(CS1 * sizeof(int));
  w.wstart = (int*)take((d.G + 2) * sizeof(int));
  w.wend = (int*)take((d.G + 2) * sizeof(int));
  w.wmulti = (int*)take((d.G + 2) * sizeof(int));
  w.wfan = (int*)take((d.G + 2) * sizeof(int));
  w.bytes = off;
  return w;
}

int grid_for(long long n, int threads = 256) {
  long long b = (n + threads - 1) / threads;
  if (b < 1) b = 1;
  if (b > 148LL * 64) b = 148LL * 64;
  return (int)b;
}

// ---- exclusive scan of int counts (three launches; in place allowed) ---------------------------

__device__ __forceinline__ long long block_scan_excl(long long v, long long* red, long long* total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  long long incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) red[wid] = incl;
  __syncthreads();
  if (wid == 0) {
    long long t = lane < nw ? red[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < nw) red[lane] = t;
  }
  __syncthreads();
  const long long before = wid == 0 ? 0 : red[wid - 1];
  *total = red[nw - 1];
  __syncthreads();  // red is reused by the caller's next call
  return before + incl - v;
}

__global__ void __launch_bounds__(SC_THREADS) scan_sums_kernel(const int* in, long long n, long long* sums) {
  __shared__ long long red[32];
  const long long b = (long long)blockIdx.x * SC_TILE + (long long)threadIdx.x * SC_VALS;
  long long s = 0;
#pragma unroll
  for (int k = 0; k < SC_VALS; ++k)
    if (b + k < n) s += in[b + k];
  long long tot;
  block_scan_excl(s, red, &tot);
  if (threadIdx.x == 0) sums[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(SC_THREADS) scan_top_kernel(long long* sums, long long n_tiles, long long* total) {
  __shared__ long long red[32];
  long long carry = 0;
  for (long long b = 0; b < n_tiles; b += SC_THREADS) {
    const long long i = b + threadIdx.x;
    const long long v = i < n_tiles ? sums[i] : 0;
    long long tot;
    const long long ex = block_scan_excl(v, red, &tot);
    if (i < n_tiles) sums[i] = carry + ex;
    carry += tot;
  }
  if (threadIdx.x == 0) *total = carry;
}

// out[0..n) = exclusive scan of in (out may be in); out[n] = total when write_total; sets
// ST_OVERFLOW when the total exceeds INT_MAX.
__global__ void __launch_bounds__(SC_THREADS) scan_tiles_kernel(const int* in, int* out, long long n,
                                                                 const long long* sums, const long long* total,
                                                                 int write_total, int* status) {
  __shared__ long long red[32];
  const long long b = (long long)blockIdx.x * SC_TILE + (long long)threadIdx.x * SC_VALS;
  int v[SC_VALS];
  long long s = 0;
#pragma unroll
  for (int k = 0; k < SC_VALS; ++k) {
    v[k] = b + k < n ? in[b + k] : 0;
    s += v[k];
  }
  long long tot;
  long long run = sums[blockIdx.x] + block_scan_excl(s, red, &tot);
#pragma unroll
  for (int k = 0; k < SC_VALS; ++k) {
    if (b + k < n) out[b + k] = (int)run;
    run += v[k];
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (*total > INT_MAX) atomicOr(status, ST_OVERFLOW);
    if (write_total) out[n] = (int)*total;
  }
}

void scan_excl(const int* in, int* out, long long n, const ScanCtx& w, bool write_total, cudaStream_t st) {
  const long long nt = sc_tiles(n > 0 ? n : 1);
  scan_sums_kernel<<<(unsigned)nt, SC_THREADS, 0, st>>>(in, n, w.sums);
  scan_top_kernel<<<1, SC_THREADS, 0, st>>>(w.sums, nt, w.total);
  scan_tiles_kernel<<<(unsigned)nt, SC_THREADS, 0, st>>>(in, out, n, w.sums, w.total, write_total ? 1 : 0,
                                                         w.status);
}

// ---- stable LSD radix sort (8-bit digits) -------------------------------------------------------

__device__ __forceinline__ unsigned rx_digit(const u64* k64, const unsigned* g32, long long i, int shift) {
  return g32 ? ((g32[i] >> shift) & 255u) : (unsigned)((k64[i] >> shift) & 255ull);
}

// hist[d * n_tiles + tile] = number of keys of the tile with digit d (g32 != null: digit of g32).
__global__ void __launch_bounds__(32 * RX_WARPS) radix_hist_kernel(const u64* k64, const unsigned* g32, long long n,
                                                                   int shift, long long n_tiles, int* hist) {
  __shared__ int cnt[RX_WARPS][256];
  const int lane = threadIdx.x & 31, wv = threadIdx.x >> 5;
  const long long tile = (long long)blockIdx.x * RX_WARPS + wv;
  if (tile >= n_tiles) return;
  for (int d = lane; d < 256; d += 32) cnt[wv][d] = 0;
  __syncwarp();
  const long long b = tile * RX_TILE, e = b + RX_TILE < n ? b + RX_TILE : n;
  for (long long i = b + lane; i < e; i += 32) atomicAdd(&cnt[wv][rx_digit(k64, g32, i, shift)], 1);
  __syncwarp();
  for (int d = lane; d < 256; d += 32) hist[(size_t)d * n_tiles + tile] = cnt[wv][d];
}

// Stable scatter of one digit pass: keys of a tile are taken in order, 32 at a time; lanes with the
// same digit get consecutive positions in lane order (match_any), the digit's base advances by
// their count.  g32 / val / the k64 outputs may be null (arrays not carried).
__global__ void __launch_bounds__(32 * RX_WARPS) radix_scatter_kernel(const u64* k64, const unsigned* g32,
                                                                      const unsigned* val, u64* k64_o,
                                                                      unsigned* g32_o, unsigned* val_o,
                                                                      int digit_of_g32, long long n, int shift,
                                                                      long long n_tiles, const int* off) {
  __shared__ int base[RX_WARPS][256];
  const int lane = threadIdx.x & 31, wv = threadIdx.x >> 5;
  const long long tile = (long long)blockIdx.x * RX_WARPS + wv;
  if (tile >= n_tiles) return;
  for (int d = lane; d < 256; d += 32) base[wv][d] = off[(size_t)d * n_tiles + tile];
  __syncwarp();
  const long long b = tile * RX_TILE, e = b + RX_TILE < n ? b + RX_TILE : n;
  const unsigned lt = (1u << lane) - 1u;
  for (long long c = b; c < e; c += 32) {
    const long long i = c + lane;
    const bool valid = i < e;
    const unsigned d = valid ? rx_digit(k64, digit_of_g32 ? g32 : nullptr, i, shift) : 256u + (unsigned)lane;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    const int rank = __popc(peers & lt);
    const int pos = valid ? base[wv][d] + rank : 0;
    __syncwarp();
    if (valid) {
      if (k64_o) k64_o[pos] = k64[i];
      if (g32_o) g32_o[pos] = g32[i];
      if (val_o) val_o[pos] = val[i];
      if (rank == 0) base[wv][d] = pos + __popc(peers);
    }
    __syncwarp();
  }
}

// Sorts n entries by (g32, k64) when g32 is given (k64's `bits64` low bits, then g32's 32 bits),
// else by k64's `bits64` low bits; ping-pongs between buffer 0 and 1 and returns the index of
// the buffer holding the result.
int radix_sort(u64* k64[2], unsigned* g32[2], unsigned* val[2], long long n, int bits64, bool with_g32, int* hist,
               const ScanCtx& w, cudaStream_t st) {
  if (n <= 1) return 0;
  const long long nt = rx_tiles(n);
  const int blocks = (int)((nt + RX_WARPS - 1) / RX_WARPS);
  int cur = 0;
  auto pass = [&](bool on_g32, int shift) {
    radix_hist_kernel<<<blocks, 32 * RX_WARPS, 0, st>>>(k64[cur], on_g32 ? g32[cur] : nullptr, n, shift, nt, hist);
    scan_excl(hist, hist, 256 * nt, w, false, st);
    radix_scatter_kernel<<<blocks, 32 * RX_WARPS, 0, st>>>(
        k64[cur], with_g32 ? g32[cur] : nullptr, val ? val[cur] : nullptr, k64[cur ^ 1],
        with_g32 ? g32[cur ^ 1] : nullptr, val ? val[cur ^ 1] : nullptr, on_g32 ? 1 : 0, n, shift, nt, hist);
    cur ^= 1;
  };
  for (int s = 0; s < bits64; s += 8) pass(false, s);
  if (with_g32)
    for (int s = 0; s < 32; s += 8) pass(true, s);
  return cur;
}

// ---- topologies -> clade hashes -----------------------------------------------------------------

__global__ void topo_parent_kernel(const int* __restrict__ left, const int* __restrict__ right,
                                   const int* __restrict__ root, long long TT, int G, int* npar, int* status) {
  const long long NN = 2LL * G - 1;
  for (long long i = gtid(); i < TT * NN; i += gstride()) {
    const long long t = i / NN;
    const int v = (int)(i - t * NN);
    const int rt = root[t];
    if (v == 0 && (rt < G || rt >= NN)) atomicOr(status, ST_BAD_TOPOLOGY);
    if (v < G) continue;
    const int c1 = left[i], c2 = right[i];
    if (c1 < 0 || c1 >= NN || c2 < 0 || c2 >= NN || c1 == c2 || c1 == v || c2 == v) {
      atomicOr(status, ST_BAD_TOPOLOGY);
      continue;
    }
    npar[t * NN + c1] = v;
    npar[t * NN + c2] = v;
  }
}

// One thread per (topology, gene leaf): climbs from the leaf while it is the second child to
// reach a node, forming that node's hash and size from its two children.
__global__ void topo_hash_kernel(const int* __restrict__ left, const int* __restrict__ right,
                                 const u64* __restrict__ leaf_hash, long long TT, int T, int G, const int* npar,
                                 int* narr, u64* nh, int* nsz) {
  const long long NN = 2LL * G - 1;
  for (long long i = gtid(); i < TT * G; i += gstride()) {
    const long long t = i / G;
    const int g = (int)(i - t * G);
    const long long f = t / T;
    const size_t base = (size_t)(t * NN);
    nh[base + g] = leaf_hash[f * G + g];
    nsz[base + g] = 1;
    int node = g;
    for (long long step = 0; step < NN; ++step) {
      const int p = npar[base + node];
      if (p < G || p >= NN) break;  // the root (-1) or a malformed parent
      __threadfence();              // this node's hash is visible before the arrival is counted
      if (atomicAdd(narr + base + p, 1) == 0) break;
      __threadfence();
      const int l = left[base + p], r = right[base + p];
      nh[base + p] = __ldcg(nh + base + l) + __ldcg(nh + base + r);
      nsz[base + p] = __ldcg(nsz + base + l) + __ldcg(nsz + base + r);
      node = p;
    }
  }
}

// Clade tables: every gene leaf (size 1, its gene index) and every internal node of every topology.
__global__ void clade_insert_kernel(const u64* __restrict__ leaf_hash, const u64* nh, const int* nsz, int F, int T,
                                    int G, int cl, u64* ckey, int* csize, int* cleaf, int* status) {
  const long long NN = 2LL * G - 1, NI = G - 1;
  const long long n_leaf = (long long)F * G, n_int = (long long)F * T * NI;
  const int mask = (1 << cl) - 1;
  for (long long i = gtid(); i < n_leaf + n_int; i += gstride()) {
    long long f;
    u64 h;
    int sz, g = -1;
    if (i < n_leaf) {
      f = i / G;
      g = (int)(i - f * G);
      h = leaf_hash[i];
      sz = 1;
    } else {
      const long long j = i - n_leaf, t = j / NI, v = G + (j - t * NI);
      f = t / T;
      h = nh[t * NN + v];
      sz = nsz[t * NN + v];
    }
    if (h == EMPTY) {
      atomicOr(status, ST_RESERVED_HASH);
      continue;
    }
    if (sz < 1 || sz > G) {  // only a malformed topology (a cycle) sums past G leaves; sizes key the waves
      atomicOr(status, ST_BAD_TOPOLOGY);
      continue;
    }
    bool fresh;
    const int s = table_insert(ckey + (f << cl), mask, h, &fresh);
    if (s < 0) {
      atomicOr(status, ST_CLADE_FULL);
      continue;
    }
    const size_t gs = (size_t)(f << cl) + s;
    if (g >= 0) {  // a leaf's size wins over an internal clade of the same hash, as on the host
      atomicExch(csize + gs, 1);
      cleaf[gs] = g;
    } else {
      atomicCAS(csize + gs, 0, sz);
    }
  }
}

// Observed splits: one per internal node of every topology, counted.
__global__ void split_insert_kernel(const int* __restrict__ left, const int* __restrict__ right, const u64* nh,
                                    int F, int T, int G, int cl, int sl, const u64* ckey, u64* skey, int* scount,
                                    int* sL, int* sH, int* status) {
  const long long NN = 2LL * G - 1, NI = G - 1;
  const int cmask = (1 << cl) - 1, smask = (1 << sl) - 1;
  for (long long j = gtid(); j < (long long)F * T * NI; j += gstride()) {
    const long long t = j / NI, v = G + (j - t * NI), f = t / T;
    const size_t base = (size_t)(t * NN);
    const int c1 = left[base + v], c2 = right[base + v];
    if (c1 < 0 || c1 >= NN || c2 < 0 || c2 >= NN) continue;  // flagged by topo_parent_kernel
    const u64 h = nh[base + v];
    const u64 ha = nh[base + c1], hb = nh[base + c2];
    const u64 lo = ha < hb ? ha : hb, hi = ha < hb ? hb : ha;
    const u64* ck = ckey + (f << cl);
    const int X = table_find(ck, cmask, h), L = table_find(ck, cmask, lo), H = table_find(ck, cmask, hi);
    if (X < 0 || L < 0 || H < 0) {
      atomicOr(status, ST_MISSING);
      continue;
    }
    bool fresh;
    const int s = table_insert(skey + (f << sl), smask, ((u64)X << 32) | (u64)L, &fresh);
    if (s < 0) {
      atomicOr(status, ST_SPLIT_FULL);
      continue;
    }
    const size_t gs = (size_t)(f << sl) + s;
    atomicAdd(scount + gs, 1);
    sL[gs] = (int)((f << cl) + L);
    sH[gs] = (int)((f << cl) + H);
  }
}

// Per clade: number of splits (and the sum of their counts when cnobs != null).
__global__ void csr_count_kernel(const u64* skey, const int* scount, int cl, int sl, long long SS, int* cnspl,
                                 int* cnobs) {
  for (long long s = gtid(); s < SS; s += gstride()) {
    const u64 k = skey[s];
    if (k == EMPTY) continue;
    const long long X = ((s >> sl) << cl) + (long long)(k >> 32);
    atomicAdd(cnspl + X, 1);
    if (cnobs) atomicAdd(cnobs + X, scount[s]);
  }
}

__global__ void csr_fill_kernel(const u64* skey, int cl, int sl, long long SS, int* ccur, int* csr) {
  for (long long s = gtid(); s < SS; s += gstride()) {
    const u64 k = skey[s];
    if (k == EMPTY) continue;
    const long long X = ((s >> sl) << cl) + (long long)(k >> 32);
    csr[atomicAdd(ccur + X, 1)] = (int)s;
  }
}

// Inserts split (lo | hi) of clade X_local (family f) with count 0 unless present.
__device__ __forceinline__ void propose(u64* skey, int* sL, int* sH, long long f, int cl, int sl, int X_local,
                                        int lo_g, int hi_g, int* status, u64* added) {
  const int lo_local = lo_g - (int)(f << cl);
  bool fresh;
  const int s = table_insert(skey + (f << sl), (1 << sl) - 1, ((u64)X_local << 32) | (u64)lo_local, &fresh);
  if (s < 0) {
    atomicOr(status, ST_SPLIT_FULL);
    return;
  }
  if (fresh) {
    const size_t gs = (size_t)(f << sl) + s;
    sL[gs] = lo_g;
    sH[gs] = hi_g;
    atomicAdd(added, 1ull);
  }
}

// One amalgamation round over the CSR snapshot (cptr / cnspl / csr of the round's start).
__global__ void amalg_kernel(const int* __restrict__ csr, const int* __restrict__ cptr,
                             const int* __restrict__ cnspl, long long CS, const u64* __restrict__ ckey,
                             const int* __restrict__ csize, int cl, int sl, u64* skey, int* sL, int* sH,
                             int* status, u64* added) {
  const long long n = cptr[CS];
  const int cmask = (1 << cl) - 1;
  for (long long e = gtid(); e < n; e += gstride()) {
    const int s = csr[e];
    const long long f = (long long)s >> sl;
    const int X_local = (int)(skey[s] >> 32);
    const int Ls = sL[s], Hs = sH[s];
    const u64* ck = ckey + (f << cl);
    for (int o = 0; o < 2; ++o) {
      const int Cs = o ? Hs : Ls, Os = o ? Ls : Hs;
      const int nc = cnspl[Cs];
      if (nc == 0) continue;
      const u64 ho = ckey[Os];
      const int s_ho = csize[Os];
      const int b0 = cptr[Cs];
      for (int j = 0; j < nc; ++j) {
        const int s2 = csr[b0 + j];
        const int L2 = sL[s2], H2 = sH[s2];
        const u64 h1 = ckey[L2], h2 = ckey[H2];
        // move h2 next to ho, keep h1
        u64 hy = h2 + ho;
        int Y = table_find(ck, cmask, hy);
        if (Y >= 0) {
          const int Yg = (int)(f << cl) + Y;
          if (csize[Yg] == csize[H2] + s_ho) {
            if (h1 < hy) propose(skey, sL, sH, f, cl, sl, X_local, L2, Yg, status, added);
            else propose(skey, sL, sH, f, cl, sl, X_local, Yg, L2, status, added);
          }
        }
        // move h1 next to ho, keep h2
        hy = h1 + ho;
        Y = table_find(ck, cmask, hy);
        if (Y >= 0) {
          const int Yg = (int)(f << cl) + Y;
          if (csize[Yg] == csize[L2] + s_ho) {
            if (h2 < hy) propose(skey, sL, sH, f, cl, sl, X_local, H2, Yg, status, added);
            else propose(skey, sL, sH, f, cl, sl, X_local, Yg, H2, status, added);
          }
        }
      }
    }
  }
}

__global__ void split_logp_kernel(const u64* skey, const int* scount, const int* cnspl, const int* cnobs, int cl,
                                  int sl, long long SS, double alpha, float* slp) {
  for (long long s = gtid(); s < SS; s += gstride()) {
    const u64 k = skey[s];
    if (k == EMPTY) continue;
    const long long X = ((s >> sl) << cl) + (long long)(k >> 32);
    const double denom = (double)cnobs[X] + alpha * (double)cnspl[X];
    slp[s] = (float)log2(((double)scount[s] + alpha) / denom);
  }
}

__global__ void occupied_kernel(const u64* ckey, long long CS, int* flag) {
  for (long long i = gtid(); i < CS; i += gstride()) flag[i] = ckey[i] != EMPTY;
}

__global__ void row_keys_kernel(const u64* ckey, const int* csize, const int* cleaf, const int* cnspl,
                                const int* pos, long long CS, int cl, u64* k64, unsigned* g32, unsigned* val) {
  for (long long i = gtid(); i < CS; i += gstride()) {
    const u64 h = ckey[i];
    if (h == EMPTY) continue;
    const int p = pos[i];
    const int lf = cleaf[i];
    k64[p] = lf >= 0 ? (u64)lf : h;
    g32[p] = ((unsigned)csize[i] << 16) | ((cnspl[i] > 1 ? 1u : 0u) << 15) | (unsigned)(i >> cl);
    val[p] = (unsigned)i;
  }
}

// Row ids, wave-start flags and per-row split counts of the sorted rows.
__global__ void rows_kernel(const unsigned* g32, const unsigned* val, long long C, const int* cnspl, int* crow,
                            int* wflag, int* rnspl) {
  for (long long r = gtid(); r < C; r += gstride()) {
    const unsigned i = val[r];
    crow[i] = (int)r;
    wflag[r] = (r == 0 || (g32[r] >> 16) != (g32[r - 1] >> 16)) ? 1 : 0;
    rnspl[r] = cnspl[i];
  }
}

// wave index of row r = (inclusive count of wave starts up to r) - 1 = wscan[r+1] - 1.
__global__ void waves_kernel(const unsigned* g32, long long C, const int* wscan, int* wstart, int* wend,
                             int* wmulti) {
  for (long long r = gtid(); r < C; r += gstride()) {
    const int w = wscan[r + 1] - 1;
    const unsigned sz = g32[r] >> 16;
    if (r == 0 || (g32[r - 1] >> 16) != sz) wstart[w] = (int)r;
    if (r == C - 1 || (g32[r + 1] >> 16) != sz) wend[w] = (int)(r + 1);
    if ((g32[r] >> 15) & 1u) atomicMin(wmulti + w, (int)r);
  }
}

__global__ void init_waves_kernel(int* wmulti, int* wfan, int n) {
  for (long long i = gtid(); i < n; i += gstride()) {
    wmulti[i] = INT_MAX;
    wfan[i] = 0;
  }
}

// ---- emission --------------------------------------------------------------------------------

__global__ void emit_rows_kernel(const unsigned* g32, const unsigned* val, long long C, long long G,
                                 const int* wscan, const int* wstart, const int* wend, const int* wmulti, int* wfan,
                                 const int* rsp, const int* cptr, const int* cnspl, const int* csr, const int* sL,
                                 const int* sH, const float* slp, const u64* ckey, const int* cleaf, const int* crow,
                                 const long long* leaf_species, int* leaf_state, long long* item_idx,
                                 long long* row_local, long long* sl_o, long long* sr_o, long long* red_o,
                                 long long* srow_o, long long* rsp_o, float* lsp_o, long long* ge2_flat,
                                 u64* child_keys) {
  for (long long r = gtid(); r < C; r += gstride()) {
    const unsigned i = val[r];
    const long long f = g32[r] & 0x7FFFu;
    const int w = wscan[r + 1] - 1;
    const int ws = wstart[w], we = wend[w];
    const int wm = wmulti[w] < we ? wmulti[w] : we;
    const int lf = cleaf[i];
    item_idx[r] = f;
    leaf_state[r] = lf >= 0 ? (int)leaf_species[f * G + lf] : -1;
    const long long loc = r - ws;
    row_local[r] = loc;
    const int e0 = rsp[r], n = cnspl[i], b0 = cptr[i];
    rsp_o[r] = e0;
    if (r == C - 1) rsp_o[C] = rsp[C];
    // this row's split slots, ordered by the smaller child's hash (insertion sort in place)
    for (int j = 0; j < n; ++j) {
      const int s = csr[b0 + j];
      const u64 key = ckey[sL[s]];
      int k = j;
      while (k > 0 && ckey[sL[(int)sl_o[e0 + k - 1]]] > key) {
        sl_o[e0 + k] = sl_o[e0 + k - 1];
        --k;
      }
      sl_o[e0 + k] = s;
    }
    for (int j = 0; j < n; ++j) {
      const int s = (int)sl_o[e0 + j];
      const int cl_row = crow[sL[s]], ch_row = crow[sH[s]];
      sl_o[e0 + j] = cl_row;
      sr_o[e0 + j] = ch_row;
      red_o[e0 + j] = loc;
      srow_o[e0 + j] = r;
      lsp_o[e0 + j] = slp[s];
      child_keys[2LL * (e0 + j)] = (u64)w * (u64)C + (u64)cl_row;
      child_keys[2LL * (e0 + j) + 1] = (u64)w * (u64)C + (u64)ch_row;
    }
    // per wave: ge2_ptr of the multi-split rows (relative to the first of them) at ge2_flat[r + w]
    if (r >= wm) {
      ge2_flat[r + w] = rsp[r] - rsp[wm];
      atomicMax(wfan + w, n);
    }
    if (r == we - 1) ge2_flat[we + w] = rsp[we] - rsp[wm];
  }
}

__global__ void wave_table_kernel(const int* wstart, const int* wend, const int* wmulti, const int* wfan,
                                  const int* rsp, const unsigned* g32, int n_waves, long long* table) {
  for (long long w = gtid(); w < n_waves; w += gstride()) {
    const int ws = wstart[w], we = wend[w];
    const int wm = wmulti[w] < we ? wmulti[w] : we;
    long long* t = table + 8 * w;
    t[0] = ws;
    t[1] = we - ws;
    t[2] = wm - ws;
    t[3] = rsp[ws];
    t[4] = rsp[we];
    t[5] = wfan[w];
    t[6] = g32[ws] >> 16;
    t[7] = (long long)wm + w;  // ge2_ptr slice start in ge2_flat
  }
}

__global__ void roots_kernel(const u64* __restrict__ leaf_hash, int F, int G, int cl, const u64* ckey,
                             const int* crow, long long* root_rows, int* status) {
  for (long long f = gtid(); f < F; f += gstride()) {
    u64 h = 0;
    for (int g = 0; g < G; ++g) h += leaf_hash[f * G + g];
    const int X = table_find(ckey + (f << cl), (1 << cl) - 1, h);
    if (X < 0) {
      atomicOr(status, ST_MISSING);
      root_rows[f] = -1;
      continue;
    }
    root_rows[f] = crow[(f << cl) + X];
  }
}

__global__ void count_distinct_kernel(const u64* k, long long n, unsigned long long* out) {
  unsigned long long c = 0;
  for (long long i = gtid(); i < n; i += gstride()) c += (i == 0 || k[i] != k[i - 1]) ? 1ull : 0ull;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0 && c) atomicAdd(out, c);
}

bool dims_ok(int F, int T, int G, int cl, int sl) {
  if (F < 1 || F > 32767 || T < 1 || G < 2 || G > 65535 || cl < 4 || cl > 30 || sl < 4 || sl > 30) return false;
  if (((long long)F << cl) >= INT_MAX || ((long long)F << sl) >= INT_MAX) return false;
  if ((long long)F * T * (2LL * G - 1) >= (1LL << 40)) return false;
  return true;
}

int launched(cudaStream_t) { return cudaGetLastError() == cudaSuccess ? KB_OK : KB_ERR_LAUNCH; }

}  // namespace

extern "C" int kb_build_workspace(int n_families, int n_topologies, int n_genes, int clade_cap_log2,
                                  int split_cap_log2, long long* bytes_out) {
  if (!bytes_out || !dims_ok(n_families, n_topologies, n_genes, clade_cap_log2, split_cap_log2)) return KB_ERR_ARG;
  const Dims d = make_dims(n_families, n_topologies, n_genes, clade_cap_log2, split_cap_log2);
  *bytes_out = (long long)carve(nullptr, d).bytes;
  return KB_OK;
}

extern "C" int kb_build_tables(const int* left, const int* right, const int* root, const unsigned long long* leaf_hash,
                               int n_families, int n_topologies, int n_genes, int amalg_rounds, double alpha,
                               int clade_cap_log2, int split_cap_log2, void* ws, long long ws_bytes,
                               long long* sizes_out, void* stream) {
  if (!left || !right || !root || !leaf_hash || !ws || !sizes_out || amalg_rounds < 0 || !(alpha > 0.0))
    return KB_ERR_ARG;
  if (!dims_ok(n_families, n_topologies, n_genes, clade_cap_log2, split_cap_log2)) return KB_ERR_ARG;
  const Dims d = make_dims(n_families, n_topologies, n_genes, clade_cap_log2, split_cap_log2);
  const Work w = carve(ws, d);
  if ((long long)w.bytes > ws_bytes) return KB_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int cl = d.cl, sl = d.sl;
  const long long TT = (long long)d.F * d.T;

  cudaMemsetAsync(w.status, 0, 8 * sizeof(int), st);
  cudaMemsetAsync(w.counters, 0, 8 * sizeof(u64), st);
  cudaMemsetAsync(w.npar, 0xFF, d.nodes * sizeof(int), st);
  cudaMemsetAsync(w.narr, 0, d.nodes * sizeof(int), st);
  cudaMemsetAsync(w.ckey, 0xFF, d.CS * sizeof(u64), st);
  cudaMemsetAsync(w.csize, 0, d.CS * sizeof(int), st);
  cudaMemsetAsync(w.cleaf, 0xFF, d.CS * sizeof(int), st);
  cudaMemsetAsync(w.skey, 0xFF, d.SS * sizeof(u64), st);
  cudaMemsetAsync(w.scount, 0, d.SS * sizeof(int), st);

  topo_parent_kernel<<<grid_for(d.nodes), 256, 0, st>>>(left, right, root, TT, d.G, w.npar, w.status);
  topo_hash_kernel<<<grid_for(TT * d.G), 256, 0, st>>>(left, right, leaf_hash, TT, d.T, d.G, w.npar, w.narr, w.nh,
                                                       w.nsz);
  clade_insert_kernel<<<grid_for((long long)d.F * d.G + d.inst), 256, 0, st>>>(leaf_hash, w.nh, w.nsz, d.F, d.T, d.G,
                                                                               cl, w.ckey, w.csize, w.cleaf, w.status);
  split_insert_kernel<<<grid_for(d.inst), 256, 0, st>>>(left, right, w.nh, d.F, d.T, d.G, cl, sl, w.ckey, w.skey,
                                                        w.scount, w.sL, w.sH, w.status);

  auto build_csr = [&](bool with_obs) {
    cudaMemsetAsync(w.cnspl, 0, (d.CS + 1) * sizeof(int), st);
    if (with_obs) cudaMemsetAsync(w.cnobs, 0, d.CS * sizeof(int), st);
    csr_count_kernel<<<grid_for(d.SS), 256, 0, st>>>(w.skey, w.scount, cl, sl, d.SS, w.cnspl,
                                                     with_obs ? w.cnobs : nullptr);
    scan_excl(w.cnspl, w.cptr, d.CS, w.scan(), true, st);
    cudaMemcpyAsync(w.ccur, w.cptr, (d.CS + 1) * sizeof(int), cudaMemcpyDeviceToDevice, st);
    csr_fill_kernel<<<grid_for(d.SS), 256, 0, st>>>(w.skey, cl, sl, d.SS, w.ccur, w.csr);
  };
  for (int r = 0; r < amalg_rounds; ++r) {
    build_csr(false);
    amalg_kernel<<<grid_for(d.SS), 256, 0, st>>>(w.csr, w.cptr, w.cnspl, d.CS, w.ckey, w.csize, cl, sl, w.skey, w.sL,
                                                 w.sH, w.status, w.counters);
  }
  build_csr(true);
  split_logp_kernel<<<grid_for(d.SS), 256, 0, st>>>(w.skey, w.scount, w.cnspl, w.cnobs, cl, sl, d.SS, alpha, w.slp);

  // rows: occupied clade slots, compacted, sorted by (size, multi, family, hash | gene index)
  occupied_kernel<<<grid_for(d.CS), 256, 0, st>>>(w.ckey, d.CS, w.rflag);
  scan_excl(w.rflag, w.rflag, d.CS, w.scan(), true, st);
  long long h_c = 0;
  cudaMemcpyAsync(&h_c, w.total, sizeof(long long), cudaMemcpyDeviceToHost, st);
  if (cudaStreamSynchronize(st) != cudaSuccess) return KB_ERR_LAUNCH;
  const long long C = h_c;
  row_keys_kernel<<<grid_for(d.CS), 256, 0, st>>>(w.ckey, w.csize, w.cleaf, w.cnspl, w.rflag, d.CS, cl, w.k64[0],
                                                  w.g32[0], w.val[0]);
  u64* k64b[2] = {w.k64[0], w.k64[1]};
  unsigned* g32b[2] = {w.g32[0], w.g32[1]};
  unsigned* valb[2] = {w.val[0], w.val[1]};
  const int cur = radix_sort(k64b, g32b, valb, C, 64, true, w.hist, w.scan(), st);
  if (cur != 0) {  // results back in buffer 0 (12 passes: always even, kept for clarity)
    cudaMemcpyAsync(w.k64[0], w.k64[cur], C * sizeof(u64), cudaMemcpyDeviceToDevice, st);
    cudaMemcpyAsync(w.g32[0], w.g32[cur], C * sizeof(unsigned), cudaMemcpyDeviceToDevice, st);
    cudaMemcpyAsync(w.val[0], w.val[cur], C * sizeof(unsigned), cudaMemcpyDeviceToDevice, st);
  }
  rows_kernel<<<grid_for(C), 256, 0, st>>>(w.g32[0], w.val[0], C, w.cnspl, w.crow, w.rwave, w.rsp);
  scan_excl(w.rwave, w.rwave, C, w.scan(), true, st);  // exclusive: wave of row r = rwave[r + 1] - 1, rwave[C] = waves
  scan_excl(w.rsp, w.rsp, C, w.scan(), true, st);
  init_waves_kernel<<<grid_for(d.G + 2), 256, 0, st>>>(w.wmulti, w.wfan, d.G + 2);
  waves_kernel<<<grid_for(C), 256, 0, st>>>(w.g32[0], C, w.rwave, w.wstart, w.wend, w.wmulti);
  int h_tail[2] = {0, 0};
  cudaMemcpyAsync(&h_tail[0], w.rwave + C, sizeof(int), cudaMemcpyDeviceToHost, st);
  cudaMemcpyAsync(&h_tail[1], w.rsp + C, sizeof(int), cudaMemcpyDeviceToHost, st);
  int h_status = 0;
  cudaMemcpyAsync(&h_status, w.status, sizeof(int), cudaMemcpyDeviceToHost, st);
  u64 h_added = 0;
  cudaMemcpyAsync(&h_added, w.counters, sizeof(u64), cudaMemcpyDeviceToHost, st);
  if (cudaStreamSynchronize(st) != cudaSuccess) return KB_ERR_LAUNCH;
  sizes_out[0] = C;
  sizes_out[1] = h_tail[1];
  sizes_out[2] = h_tail[0];
  sizes_out[3] = h_status;
  sizes_out[4] = (long long)h_added;
  return launched(st);
}

extern "C" int kb_build_emit_scratch(long long n_splits, long long* bytes_out) {
  if (n_splits < 0 || !bytes_out) return KB_ERR_ARG;
  const long long n = 2 * n_splits;
  *bytes_out = 2 * ((n * 8 + 255) / 256 * 256) + (256 * rx_tiles(n > 0 ? n : 1) + 1) * 4 + 256;
  return KB_OK;
}

extern "C" int kb_build_emit(const void* ws, const unsigned long long* leaf_hash, const long long* leaf_species,
                             int n_families, int n_topologies, int n_genes, int clade_cap_log2, int split_cap_log2,
                             long long n_rows, long long n_splits, long long n_waves, int* leaf_state,
                             long long* item_idx, long long* root_row_ids, long long* row_local, long long* sl,
                             long long* sr, long long* reduce_idx, long long* split_row, long long* row_split_ptr,
                             float* log_split_probs, long long* ge2_flat, long long* wave_table, void* scratch,
                             long long scratch_bytes,
                             long long* k_children_out, void* stream) {
  if (!ws || !leaf_hash || !leaf_species || !k_children_out) return KB_ERR_ARG;
  if (!dims_ok(n_families, n_topologies, n_genes, clade_cap_log2, split_cap_log2)) return KB_ERR_ARG;
  if (n_rows < 1 || n_splits < 0 || n_waves < 1 || n_waves > n_genes + 1) return KB_ERR_ARG;
  long long need = 0;
  kb_build_emit_scratch(n_splits, &need);
  if (scratch_bytes < need || !scratch) return KB_ERR_ARG;
  const Dims d = make_dims(n_families, n_topologies, n_genes, clade_cap_log2, split_cap_log2);
  // the workspace is only read here, apart from the per-wave fan-out maxima and the scan scratch
  const Work w = carve(const_cast<void*>(ws), d);
  cudaStream_t st = (cudaStream_t)stream;
  const long long C = n_rows, N = n_splits, n2 = 2 * N;
  char* sc = static_cast<char*>(scratch);
  const size_t kb = (size_t)((n2 * 8 + 255) / 256 * 256);
  u64* keys[2] = {reinterpret_cast<u64*>(sc), reinterpret_cast<u64*>(sc + kb)};
  int* hist = reinterpret_cast<int*>(sc + 2 * kb);
  unsigned long long* kcount =
      reinterpret_cast<unsigned long long*>(sc + 2 * kb + ((256 * rx_tiles(n2 > 0 ? n2 : 1) + 1) * 4 + 7) / 8 * 8);

  cudaMemsetAsync(w.wfan, 0, (d.G + 2) * sizeof(int), st);
  emit_rows_kernel<<<grid_for(C), 256, 0, st>>>(w.g32[0], w.val[0], C, d.G, w.rwave, w.wstart, w.wend, w.wmulti,
                                                w.wfan, w.rsp, w.cptr, w.cnspl, w.csr, w.sL, w.sH, w.slp, w.ckey,
                                                w.cleaf, w.crow, leaf_species, leaf_state, item_idx, row_local, sl,
                                                sr, reduce_idx, split_row, row_split_ptr, log_split_probs,
                                                ge2_flat, keys[0]);
  wave_table_kernel<<<grid_for(n_waves), 256, 0, st>>>(w.wstart, w.wend, w.wmulti, w.wfan, w.rsp, w.g32[0],
                                                       (int)n_waves, wave_table);
  roots_kernel<<<grid_for(d.F), 256, 0, st>>>(leaf_hash, d.F, d.G, d.cl, w.ckey, w.crow, root_row_ids, w.status);
  // distinct (wave, child row) pairs
  int bits = 0;
  while (bits < 64 && ((unsigned long long)n_waves * (unsigned long long)C) >> bits) ++bits;
  bits = (bits + 7) / 8 * 8;
  unsigned* none[2] = {nullptr, nullptr};
  const int cur = radix_sort(keys, none, nullptr, n2, bits, false, hist, w.scan(), st);
  cudaMemsetAsync(kcount, 0, sizeof(unsigned long long), st);
  if (n2 > 0) count_distinct_kernel<<<grid_for(n2), 256, 0, st>>>(keys[cur], n2, kcount);
  int h_status = 0;
  unsigned long long h_k = 0;
  cudaMemcpyAsync(&h_k, kcount, sizeof(h_k), cudaMemcpyDeviceToHost, st);
  cudaMemcpyAsync(&h_status, w.status, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (cudaStreamSynchronize(st) != cudaSuccess) return KB_ERR_LAUNCH;
  k_children_out[0] = (long long)h_k;
  k_children_out[1] = h_status;
  return launched(st);
}

// =================================================================================================
// The engine's schedule from a row-ordered layout (the device counterpart of engine.build_plan):
// dependency levels (level 0: rows without splits; else 1 + the deepest child level), the rows in
// (level, row) order with their splits, distinct child rows per level, and the dataflow arrays
// (distinct (parent, child) pairs as CSR by parent and by child, ready rows).
// =================================================================================================

namespace {

struct PlanWork {
  int* status;
  u64* counters;  // [0] max level
  long long* total;
  long long* sums;
  int* level;     // [C]
  u64* k64[2];    // [M] sort keys (M = max(C, 2N))
  unsigned* val[2];
  int* hist;
  int* pos;       // [C]
  int* cnt;       // [C+1]
  int* flag;      // [M+1]
  u64* pairs;     // [2N] distinct (parent, child) keys
  int* cnt_p;     // [C+1]
  int* cnt_c;     // [C+1]
  int* lvrows;    // [C+1]
  int* lvkids;    // [C]
  size_t bytes;
  ScanCtx scan() const { return ScanCtx{sums, total, status}; }
};

PlanWork carve_plan(void* base, long long C, long long N) {
  PlanWork w{};
  size_t off = 0;
  char* b = static_cast<char*>(base);
  auto take = [&](size_t n) -> void* {
    off = (off + 255) & ~size_t(255);
    void* p = b ? b + off : nullptr;
    off += n;
    return p;
  };
  const long long M = (2 * N > C ? 2 * N : C);
  w.status = (int*)take(8 * sizeof(int));
  w.counters = (u64*)take(8 * sizeof(u64));
  w.total = (long long*)take(4 * sizeof(long long));
  w.sums = (long long*)take((sc_tiles(M + 1) + 1) * sizeof(long long));
  w.level = (int*)take(C * sizeof(int));
  for (int i = 0; i < 2; ++i) {
    w.k64[i] = (u64*)take(M * sizeof(u64));
    w.val[i] = (unsigned*)take(M * sizeof(unsigned));
  }
  w.hist = (int*)take((256 * rx_tiles(M) + 1) * sizeof(int));
  w.pos = (int*)take(C * sizeof(int));
  w.cnt = (int*)take((C + 1) * sizeof(int));
  w.flag = (int*)take((M + 1) * sizeof(int));
  w.pairs = (u64*)take((2 * N + 1) * sizeof(u64));
  w.cnt_p = (int*)take((C + 1) * sizeof(int));
  w.cnt_c = (int*)take((C + 1) * sizeof(int));
  w.lvrows = (int*)take((C + 1) * sizeof(int));
  w.lvkids = (int*)take(C * sizeof(int));
  w.bytes = off;
  return w;
}

int bits_for(unsigned long long v) {  // bits to hold values < v, rounded up to whole digits
  int b = 0;
  while (b < 64 && (v - 1) >> b) ++b;
  return (b + 7) / 8 * 8;
}

// Every split's parent and child rows in [0, C), each wave's parents in increasing row order
// (ST_MISSING otherwise).
__global__ void plan_check_kernel(const long long* par, const long long* sl, const long long* sr, long long N,
                                  long long C, int* status) {
  for (long long i = gtid(); i < N; i += gstride()) {
    const long long p = par[i], l = sl[i], r = sr[i];
    if (p < 0 || p >= C || l < 0 || l >= C || r < 0 || r >= C || (i > 0 && par[i - 1] > p))
      atomicOr(status, ST_MISSING);
  }
}

__global__ void level_wave_kernel(const long long* __restrict__ par, const long long* __restrict__ sl,
                                  const long long* __restrict__ sr, long long b, long long e, int* level) {
  for (long long i = b + gtid(); i < e; i += gstride()) {
    const int lv = max(__ldcg(level + sl[i]), __ldcg(level + sr[i])) + 1;
    atomicMax(level + par[i], lv);
  }
}

__global__ void level_keys_kernel(const int* level, long long C, u64* k, unsigned* v, int* lvrows, u64* maxlv) {
  unsigned long long m = 0;
  for (long long r = gtid(); r < C; r += gstride()) {
    const int lv = level[r];
    k[r] = (u64)lv;
    v[r] = (unsigned)r;
    atomicAdd(lvrows + lv, 1);
    m = m > (unsigned long long)lv ? m : (unsigned long long)lv;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long y = __shfl_xor_sync(0xffffffffu, m, o);
    m = m > y ? m : y;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(maxlv, m);
}

__global__ void level_rows_kernel(const unsigned* v, long long C, const long long* rsp, int* rows, int* pos, int* cnt) {
  for (long long q = gtid(); q < C; q += gstride()) {
    const unsigned r = v[q];
    rows[q] = (int)r;
    pos[r] = (int)q;
    cnt[q] = (int)(rsp[r + 1] - rsp[r]);
  }
}

__global__ void widen_kernel(const int* in, long long n, long long* out) {
  for (long long i = gtid(); i < n; i += gstride()) out[i] = in[i];
}

__global__ void level_gather_kernel(const int* rows, long long C, const long long* rsp, const long long* split_ptr,
                                    const long long* sl, const long long* sr, const float* lsp, long long* sl_o,
                                    long long* sr_o, float* lsp_o) {
  for (long long q = gtid(); q < C; q += gstride()) {
    const long long r = rows[q];
    const long long b = rsp[r], n = rsp[r + 1] - b, d = split_ptr[q];
    for (long long j = 0; j < n; ++j) {
      sl_o[d + j] = sl[b + j];
      sr_o[d + j] = sr[b + j];
      lsp_o[d + j] = lsp[b + j];
    }
  }
}

// keys[2i] = hi(i) * C + sl[i], keys[2i+1] = hi(i) * C + sr[i], hi = level of the parent (by_level)
// or the parent row itself
__global__ void child_keys_kernel(const long long* par, const long long* sl, const long long* sr, long long N,
                                  long long C, const int* level, u64* keys) {
  for (long long i = gtid(); i < N; i += gstride()) {
    const u64 hi = level ? (u64)level[par[i]] : (u64)par[i];
    keys[2 * i] = hi * (u64)C + (u64)sl[i];
    keys[2 * i + 1] = hi * (u64)C + (u64)sr[i];
  }
}

__global__ void distinct_flags_kernel(const u64* k, long long n, int* flag) {
  for (long long i = gtid(); i < n; i += gstride()) flag[i] = (i == 0 || k[i] != k[i - 1]) ? 1 : 0;
}

// cnt[hi] += number of flagged keys with high part hi; the keys are sorted, so the lanes of a warp
// mostly share hi: one atomic per distinct hi per warp.
__global__ void count_by_hi_kernel(const u64* k, const int* flag, long long n, long long C, int* cnt) {
  const long long n_pad = (n + 31) / 32 * 32;
  for (long long i = gtid(); i < n_pad; i += gstride()) {
    const bool valid = i < n;
    const long long hi = valid ? (long long)(k[i] / (u64)C) : -1;
    const int f = valid ? flag[i] : 0;
    const unsigned peers = __match_any_sync(0xffffffffu, hi);
    const unsigned hits = __ballot_sync(0xffffffffu, f != 0) & peers;
    if (valid && (threadIdx.x & 31) == __ffs(peers) - 1 && hits) atomicAdd(cnt + hi, __popc(hits));
  }
}

// distinct keys (flag[i] == 1 at position pos[i] of the exclusive scan) -> out
__global__ void compact_keys_kernel(const u64* k, const int* flag_scanned, long long n, u64* out) {
  for (long long i = gtid(); i < n; i += gstride()) {
    const int p = flag_scanned[i];
    if (i == 0 || k[i] != k[i - 1]) out[p] = k[i];
  }
}

// pairs sorted by (parent, child): child_idx, counts per parent; and the swapped keys for the
// by-child order
__global__ void pairs_kernel(const u64* pairs, long long P, long long C, int* child_idx, int* cnt_p, int* cnt_c,
                             u64* swapped) {
  for (long long k = gtid(); k < P; k += gstride()) {
    const u64 key = pairs[k];
    const long long p = (long long)(key / (u64)C), c = (long long)(key % (u64)C);
    child_idx[k] = (int)c;
    atomicAdd(cnt_p + p, 1);
    atomicAdd(cnt_c + c, 1);
    swapped[k] = (u64)c * (u64)C + (u64)p;
  }
}

__global__ void low_part_kernel(const u64* k, long long n, long long C, int* out) {
  for (long long i = gtid(); i < n; i += gstride()) out[i] = (int)(k[i] % (u64)C);
}

__global__ void zero_flags_kernel(const int* cnt, long long C, int* flag, int* dep) {
  for (long long r = gtid(); r < C; r += gstride()) {
    flag[r] = cnt[r] == 0 ? 1 : 0;
    if (dep) dep[r] = cnt[r];
  }
}

__global__ void compact_rows_kernel(const int* cnt, const int* flag_scanned, long long C, int* out) {
  for (long long r = gtid(); r < C; r += gstride())
    if (cnt[r] == 0) out[flag_scanned[r]] = (int)r;
}

}  // namespace

extern "C" int kb_plan_workspace(long long n_rows, long long n_splits, long long* bytes_out) {
  if (n_rows < 1 || n_splits < 0 || !bytes_out || n_rows >= INT_MAX || 2 * n_splits >= INT_MAX) return KB_ERR_ARG;
  *bytes_out = (long long)carve_plan(nullptr, n_rows, n_splits).bytes;
  return KB_OK;
}

extern "C" int kb_plan_build(long long n_rows, long long n_splits, int n_waves, const long long* wave_split_ptr,
                             const long long* split_row, const long long* sl, const long long* sr, const float* lsp,
                             const long long* row_split_ptr, void* ws, long long ws_bytes, int* rows,
                             long long* split_ptr, long long* sl_lv, long long* sr_lv, float* lsp_lv, int* dep0,
                             int* ready0, long long* par_ptr, int* par_idx, int* dep_b, int* ready_b,
                             long long* child_ptr, int* child_idx, long long* level_ptr, long long* children,
                             long long* sizes_out, void* stream) {
  if (n_rows < 1 || n_splits < 0 || n_waves < 1 || !wave_split_ptr || !ws || !sizes_out || !level_ptr || !children)
    return KB_ERR_ARG;
  if (n_rows >= INT_MAX || 2 * n_splits >= INT_MAX) return KB_ERR_SIZE;
  const long long C = n_rows, N = n_splits, M2 = 2 * N;
  const PlanWork w = carve_plan(ws, C, N);
  if ((long long)w.bytes > ws_bytes) return KB_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const ScanCtx sc = w.scan();
  cudaMemsetAsync(w.status, 0, 8 * sizeof(int), st);
  cudaMemsetAsync(w.counters, 0, 8 * sizeof(u64), st);
  cudaMemsetAsync(w.level, 0, C * sizeof(int), st);
  cudaMemsetAsync(w.lvrows, 0, (C + 1) * sizeof(int), st);
  cudaMemsetAsync(w.lvkids, 0, C * sizeof(int), st);
  cudaMemsetAsync(w.cnt_p, 0, (C + 1) * sizeof(int), st);
  cudaMemsetAsync(w.cnt_c, 0, (C + 1) * sizeof(int), st);
  if (N > 0) plan_check_kernel<<<grid_for(N), 256, 0, st>>>(split_row, sl, sr, N, C, w.status);
  int h_bad = 0;
  cudaMemcpyAsync(&h_bad, w.status, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (cudaStreamSynchronize(st) != cudaSuccess) return KB_ERR_LAUNCH;
  if (h_bad) return KB_ERR_ARG;
  // levels, one launch per wave of the layout (children lie in earlier waves)
  for (int v = 0; v < n_waves; ++v) {
    const long long b = wave_split_ptr[v], e = wave_split_ptr[v + 1];
    if (b < 0 || e > N || b > e) return KB_ERR_ARG;
    if (e > b) level_wave_kernel<<<grid_for(e - b), 256, 0, st>>>(split_row, sl, sr, b, e, w.level);
  }
  level_keys_kernel<<<grid_for(C), 256, 0, st>>>(w.level, C, w.k64[0], w.val[0], w.lvrows, w.counters);
  u64 h_maxlv = 0;
  cudaMemcpyAsync(&h_maxlv, w.counters, sizeof(u64), cudaMemcpyDeviceToHost, st);
  if (cudaStreamSynchronize(st) != cudaSuccess) return KB_ERR_LAUNCH;
  const long long n_levels = (long long)h_maxlv + 1;
  if (n_levels > n_waves) return KB_ERR_ARG;  // a level never exceeds the wave count of a valid layout
  u64* kb[2] = {w.k64[0], w.k64[1]};
  unsigned* vb[2] = {w.val[0], w.val[1]};
  unsigned* none[2] = {nullptr, nullptr};
  int cur = radix_sort(kb, none, vb, C, bits_for((unsigned long long)n_levels), false, w.hist, sc, st);
  level_rows_kernel<<<grid_for(C), 256, 0, st>>>(w.val[cur], C, row_split_ptr, rows, w.pos, w.cnt);
  scan_excl(w.cnt, w.cnt, C, sc, true, st);
  widen_kernel<<<grid_for(C + 1), 256, 0, st>>>(w.cnt, C + 1, split_ptr);
  level_gather_kernel<<<grid_for(C), 256, 0, st>>>(rows, C, row_split_ptr, split_ptr, sl, sr, lsp, sl_lv, sr_lv, lsp_lv);
  scan_excl(w.lvrows, w.lvrows, n_levels, sc, true, st);  // level_ptr
  // distinct child rows per level
  long long P = 0;
  if (M2 > 0) {
    child_keys_kernel<<<grid_for(N), 256, 0, st>>>(split_row, sl, sr, N, C, w.level, w.k64[0]);
    cur = radix_sort(kb, none, nullptr, M2, bits_for((unsigned long long)n_levels * (unsigned long long)C), false,
                     w.hist, sc, st);
    distinct_flags_kernel<<<grid_for(M2), 256, 0, st>>>(w.k64[cur], M2, w.flag);
    count_by_hi_kernel<<<grid_for(M2), 256, 0, st>>>(w.k64[cur], w.flag, M2, C, w.lvkids);
    // distinct (parent, child) pairs, sorted by parent then child
    child_keys_kernel<<<grid_for(N), 256, 0, st>>>(split_row, sl, sr, N, C, nullptr, w.k64[0]);
    cur = radix_sort(kb, none, nullptr, M2, bits_for((unsigned long long)C * (unsigned long long)C), false, w.hist,
                     sc, st);
    distinct_flags_kernel<<<grid_for(M2), 256, 0, st>>>(w.k64[cur], M2, w.flag);
    scan_excl(w.flag, w.flag, M2, sc, true, st);
    compact_keys_kernel<<<grid_for(M2), 256, 0, st>>>(w.k64[cur], w.flag, M2, w.pairs);
    int h_p = 0;
    cudaMemcpyAsync(&h_p, w.flag + M2, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) return KB_ERR_LAUNCH;
    P = h_p;
    // by parent: child_idx, counts; by child: parents
    pairs_kernel<<<grid_for(P), 256, 0, st>>>(w.pairs, P, C, child_idx, w.cnt_p, w.cnt_c, w.k64[0]);
    cur = radix_sort(kb, none, nullptr, P, bits_for((unsigned long long)C * (unsigned long long)C), false, w.hist, sc,
                     st);
    low_part_kernel<<<grid_for(P), 256, 0, st>>>(w.k64[cur], P, C, par_idx);
  }
  // dep0 / child_ptr from the per-parent counts, dep_b / par_ptr from the per-child counts
  zero_flags_kernel<<<grid_for(C), 256, 0, st>>>(w.cnt_p, C, w.flag, dep0);
  scan_excl(w.flag, w.flag, C, sc, true, st);
  compact_rows_kernel<<<grid_for(C), 256, 0, st>>>(w.cnt_p, w.flag, C, ready0);
  int h_r0 = 0;
  cudaMemcpyAsync(&h_r0, w.flag + C, sizeof(int), cudaMemcpyDeviceToHost, st);
  scan_excl(w.cnt_p, w.cnt_p, C, sc, true, st);
  widen_kernel<<<grid_for(C + 1), 256, 0, st>>>(w.cnt_p, C + 1, child_ptr);
  zero_flags_kernel<<<grid_for(C), 256, 0, st>>>(w.cnt_c, C, w.flag, dep_b);
  scan_excl(w.flag, w.flag, C, sc, true, st);
  compact_rows_kernel<<<grid_for(C), 256, 0, st>>>(w.cnt_c, w.flag, C, ready_b);
  int h_rb = 0;
  cudaMemcpyAsync(&h_rb, w.flag + C, sizeof(int), cudaMemcpyDeviceToHost, st);
  scan_excl(w.cnt_c, w.cnt_c, C, sc, true, st);
  widen_kernel<<<grid_for(C + 1), 256, 0, st>>>(w.cnt_c, C + 1, par_ptr);
  // host lists: level_ptr [n_levels + 1], children per level [n_levels]
  int* h_lv = new int[n_levels + 1];
  int* h_kids = new int[n_levels];
  cudaMemcpyAsync(h_lv, w.lvrows, (n_levels + 1) * sizeof(int), cudaMemcpyDeviceToHost, st);
  cudaMemcpyAsync(h_kids, w.lvkids, n_levels * sizeof(int), cudaMemcpyDeviceToHost, st);
  int h_status = 0;
  cudaMemcpyAsync(&h_status, w.status, sizeof(int), cudaMemcpyDeviceToHost, st);
  const bool ok = cudaStreamSynchronize(st) == cudaSuccess;
  if (ok) {
    for (long long l = 0; l <= n_levels; ++l) level_ptr[l] = h_lv[l];
    for (long long l = 0; l < n_levels; ++l) children[l] = M2 > 0 ? h_kids[l] : 0;
  }
  delete[] h_lv;
  delete[] h_kids;
  if (!ok) return KB_ERR_LAUNCH;
  sizes_out[0] = n_levels;
  sizes_out[1] = P;
  sizes_out[2] = h_r0;
  sizes_out[3] = h_rb;
  sizes_out[4] = h_status;
  return launched(st);
}
