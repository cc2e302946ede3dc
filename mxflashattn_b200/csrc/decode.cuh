// decode.cuh -- split-KV paged decode attention for sm_100a.
//
// One CTA per (sequence b, KV head, query-row group, split z).  All query
// rows that share the KV head (GQ heads x Sq query positions, up to 16 per
// group) are packed into the N dimension of a swapped tensor-core product,
// so every paged K/V row is read from HBM once per CTA:
//
//   S^T[16 tok, 8 rows] = K[16 tok, D] . Q^T[D, 8 rows]          (m16n8k16)
//   O^T[D, 8 rows]     += V^T[D, 16 tok] . P[16 tok, 8 rows]       (m16n8k16)
//
// Warp 4 is the producer: it resolves the block table and streams 16-token
// tiles of K and V into a ring of shared-memory slots -- one TMA box per
// 64-column block when the page size is a multiple of 16, cp.async row
// gathers otherwise -- and each slot's mbarrier counts the bytes in.  Warps
// 0-3 consume tiles round-robin, run an online softmax in the log2 domain
// (row max by warp shuffles across the 8 token groups), and merge their
// (m, l, O) states through shared memory at the end.  A split writes the
// unnormalised partial state (o, m, d) for the combine kernel; a single-split
// launch writes the normalised output (and LSE) directly.
//
// Reference behaviour followed: the split geometry and partial-state
// contract of paged_decode_v3 / split_combine (csrc_native/m1_kernel.cpp:
// 563-577, 846-853, 862-888); the attention math of mxflashattn/reference.py.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace mxfa {

struct DecodeParams {
  const void* q;         // [B, Sq, HQ, D]
  const void* k;         // paged [P, PS, HKV, D] or dense [B, PS, HKV, D]
  const void* v;
  const int* bt;         // [B, BTW] or nullptr (dense: page of batch b is b)
  const int* seqlens;    // [B] cached length before this call
  void* out;             // direct mode: [B, Sq, HQ, D]
  float* lse;            // direct mode, optional: [B, Sq, HQ]
  float* ows;            // split mode when non-null: [rows, NP, D] (rows = B*Sq*HQ)
  float* mdws;           // split mode: [rows, NP, 2]
  int B, Sq, HQ, HKV, PS, BTW, P;
  int GQ;                // HQ / HKV
  int append_len;        // total length = seqlens[b] + append_len
  int NP, c_len;         // splits; chunk z covers [z*c_len, (z+1)*c_len)
  int causal;
  float scale_log2;      // softmax_scale * log2(e)
  // TMA map shape: 3 = one box per 64-column block of K or V; 4 = one box per
  // K or V tile; 5 = one box for the whole K+V tile (tmk then spans both
  // caches, V at the lower address first when kv_swap)
  int kv_map;
  int kv_swap;
  // Single-launch split (optional, split mode only): one counter per
  // (sequence, KV head, row group), zero on entry.  The last of the NP
  // split CTAs of a unit merges the unit's partials into out / lse and
  // resets its counter to zero.
  unsigned* counters;
  // FP8 (e4m3) caches: dequantised value = stored * scale.  k_scale is folded
  // into scale_log2 by the launcher; v_scale multiplies the output.
  float v_scale;
  // Context-parallel exchange (optional, with counters): instead of writing
  // out / lse, the merging CTA of a unit publishes its (O, LSE) records,
  // tagged with the step, into the exchange buffer of every rank (peer
  // memory).  With cp_merge the same CTA then waits (bounded) until every
  // rank's records of its unit carry the step's tag, merges the unit's rows
  // into out / lse, and the last unit advances the epoch; the launcher sets
  // it only when every unit's merging CTA can wait while the rest of the
  // grid still finds room, and otherwise cp_merge_kernel on each rank
  // completes the merge.
  const unsigned long long* cp_bufs;  // [cp_world] exchange-buffer bases; [cp_rank] is local
  int cp_rank, cp_world;
  int cp_merge;
  // Length order (optional, 1 < B <= kRankMaxBatch): order[y] is the
  // sequence that grid row y runs, longest first, as length_order_kernel
  // writes it once per step for every layer.  Without it each CTA ranks the
  // lengths itself.  Only the schedule depends on it: lengths are always
  // read from seqlens.
  const int* order;
  // Fused append (optional): append_len new tokens per sequence, [B, append_len, HKV, D],
  // written into the cache by the CTA that reads them (one query-row group only).
  const void* k_new;
  const void* v_new;
};

constexpr int kDecConsumerWarps = 4;
constexpr int kRankMaxBatch = 512;  // batches up to this size are dispatched longest-first
constexpr int kDecThreads = (kDecConsumerWarps + 1) * 32;
constexpr int kTileTok = 16;

// Per-instantiation occupancy.  Several CTAs per SM overlap one CTA's
// start-up and final merge with the others' streaming, which measured worth
// more than a deeper ring: the shared-memory budget (~192 KB of ring per SM)
// is split over as many CTAs as the register file allows.
//   HD=128, 8 query rows : 3 CTAs x 8 slots  (64 KB ring each, <=136 regs)
//   HD=128, 16 query rows: 2 CTAs x 12 slots (96 KB)
//   HD=64,  8 query rows : 4 CTAs x 12 slots (48 KB, <=102 regs)
//   HD=64,  16 query rows: 3 CTAs x 16 slots (64 KB)
template <int HD, int NT, bool kFp8 = false>
struct DecodeCfg {
  static constexpr int kCtasPerSm =
      kFp8 ? (NT == 1 ? 4 : 2) : (HD == 128 ? (NT == 1 ? 3 : 2) : (NT == 1 ? 4 : 3));
  static constexpr int kElemBytes = kFp8 ? 1 : 2;
  static constexpr int kRowBytes = HD * kElemBytes;      // one cached row of one head
  static constexpr int kRowChunks = kRowBytes / 16;      // 16-byte chunks per row
  static constexpr int kDBlk = kRowBytes / 128;          // 128-byte column blocks per row
  static constexpr int kBlkBytes = kTileTok * 128;       // one column block of one tile: 2 KB
  static constexpr int kTileBytes = kTileTok * kRowBytes;  // K (or V) bytes of one tile
  static constexpr int kSlotBytes = 2 * kTileBytes;      // K + V
  static constexpr int kSlots = (192 * 1024 / kCtasPerSm) / kSlotBytes / 4 * 4;  // multiple of the consumer count
  static constexpr int kRingBytes = kSlots * kSlotBytes;
  static constexpr int kSmemBytes = kRingBytes + 2 * kSlots * 8 + 1024;
  static_assert(kDBlk >= 1, "rows narrower than one 128-byte swizzle block are not supported");
};

// Merge scratch laid over the ring once all tiles are consumed.
template <int HD, int NT>
struct DecodeMerge {
  static constexpr int kCols = 8 * NT;
  static constexpr int kStride = HD + 4;  // padded row: conflict-free fragment stores
  static constexpr int kOBytes = kDecConsumerWarps * kCols * kStride * 4;
  static constexpr int kBytes = kOBytes + 2 * kDecConsumerWarps * kCols * 4;
};

// Physical slot row (page * PS + offset) of 16-token tile t of sequence b,
// read from the block table; 0 past the last tile.  A page index past the
// table or a physical page outside the cache is flagged and redirected (the
// last table column, or row P*PS which lies past the tensor so TMA fills the
// box with zeros and reads nothing).
__device__ __forceinline__ int tile_slot_row(const DecodeParams& p, int b, int tile0, int ntiles, int t) {
  if (t >= ntiles) return 0;
  const int pos = tile0 + t * kTileTok;
  int page = pos / p.PS;
  int phys = b;
  if (p.bt != nullptr) {
    if (page >= p.BTW) {
      raise_flag(MXFA_FLAG_TABLE_TOO_NARROW);
      page = p.BTW - 1;
    }
    phys = p.bt[static_cast<size_t>(b) * p.BTW + page];
  }
  if (phys < 0 || phys >= p.P) {
    raise_flag(MXFA_FLAG_PAGE_OUT_OF_RANGE);
    phys = p.P;
  }
  return phys * p.PS + (pos % p.PS);
}

// Exchange buffer of a context-parallel group (one per rank, allocated zeroed;
// peers map it through CUDA IPC).  Every step (call) advances a device-side
// epoch e and uses half e % 2 of the records, so a rank that is one step
// ahead never overwrites what a slower rank still reads:
//   [0, 256)   header: epoch (u32), merges done (u32)
//   records    [2][world][rows][D + 2] u64 words: (tag e + 1) << 32 | value
//              bits; words 0..D-1 the normalised O, word D the natural-log
//              LSE, word D+1 padding (rows stay 16-byte aligned)
// Each word carries its own step tag and is stored and loaded as one 64-bit
// access (single-copy atomic), so a reader that sees the tag sees the value:
// no flag, and no fence between the records and a flag, is needed.
struct CpLayout {
  size_t records, record_half, bytes;
};
__host__ __device__ inline CpLayout cp_layout(int world, int rows, int D) {
  CpLayout l;
  l.records = 256;
  l.record_half = static_cast<size_t>(world) * rows * (D + 2) * 8;
  l.bytes = l.records + 2 * l.record_half;
  return l;
}

__device__ __forceinline__ uint64_t cp_word(float v, unsigned tag) {
  return (static_cast<uint64_t>(tag) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void st_words2(uint64_t* p, uint64_t a, uint64_t b) {
  asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_words2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Rows of one split's partial output, loaded as this lane's HD/32 columns.
template <int HD>
__device__ __forceinline__ void load_partial(const float* src, float (&o)[HD / 32]) {
  if constexpr (HD / 32 == 4) {
    const float4 o4 = __ldcg(reinterpret_cast<const float4*>(src));
    o[0] = o4.x; o[1] = o4.y; o[2] = o4.z; o[3] = o4.w;
  } else {
    const float2 o2 = __ldcg(reinterpret_cast<const float2*>(src));
    o[0] = o2.x; o[1] = o2.y;
  }
}

// The reduction behind merge_split_row and merge_split_row_publish: M, L and
// the unnormalised sum of the weighted partial rows (this lane's columns).
// For NP <= 64 every lane loads the (m, d) pairs of splits lane and lane+32
// once, in the same round as the first 8 partial rows; the weights reach the
// other lanes by shuffle (-1 marks a split with nothing to add), and the
// remaining partial rows follow 8 at a time.  A merge is then ceil(NP/8)
// dependent L2 round trips instead of two more for the two passes over the
// pairs.  The arithmetic and its order are those of the loop form below
// (used for NP > 64, and always when kChunked is false): the same M, L and
// accumulation, bit for bit.
template <int HD, bool kChunked = true>
__device__ __forceinline__ void merge_split_core(const float* ows, const float* mdws, int r, int NP, int lane,
                                                 float (&acc)[HD / 32], float& M_out, float& L_out) {
  constexpr int kPer = HD / 32;
  constexpr int kChunk = 8;
  const float2* md = reinterpret_cast<const float2*>(mdws + static_cast<size_t>(r) * NP * 2);
  const float* src = ows + static_cast<size_t>(r) * NP * HD + lane * kPer;
#pragma unroll
  for (int j = 0; j < kPer; ++j) acc[j] = 0.f;
  float M = -INFINITY, L = 0.f;
  if (kChunked && NP <= 64) {
    float2 v0 = make_float2(-INFINITY, 0.f), v1 = make_float2(-INFINITY, 0.f);
    if (lane < NP) v0 = __ldcg(md + lane);
    if (lane + 32 < NP) v1 = __ldcg(md + lane + 32);
    float o[kChunk][kPer];
#pragma unroll
    for (int c = 0; c < kChunk; ++c)
      if (c < NP) load_partial<HD>(src + static_cast<size_t>(c) * HD, o[c]);
    const bool ok0 = v0.x > -INFINITY && v0.y > 0.f;
    const bool ok1 = v1.x > -INFINITY && v1.y > 0.f;
    if (ok0) M = fmaxf(M, v0.x);
    if (ok1) M = fmaxf(M, v1.x);
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
    float w0 = -1.f, w1 = -1.f;
    if (M != -INFINITY) {
      if (ok0) {
        w0 = fast_exp2(v0.x - M);
        L += v0.y * w0;
      }
      if (ok1) {
        w1 = fast_exp2(v1.x - M);
        L += v1.y * w1;
      }
    }
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) L += __shfl_xor_sync(0xffffffffu, L, sh);
    if (M != -INFINITY) {
      for (int base = 0; base < NP; base += kChunk) {
        if (base > 0) {
#pragma unroll
          for (int c = 0; c < kChunk; ++c)
            if (base + c < NP) load_partial<HD>(src + static_cast<size_t>(base + c) * HD, o[c]);
        }
#pragma unroll
        for (int c = 0; c < kChunk; ++c) {
          const int pz = base + c;
          // every lane takes part in both shuffles (pz is warp-uniform)
          const float wa = __shfl_sync(0xffffffffu, w0, pz & 31);
          const float wb = __shfl_sync(0xffffffffu, w1, pz & 31);
          const float w = pz < 32 ? wa : wb;
          if (pz < NP && w >= 0.f) {
#pragma unroll
            for (int j = 0; j < kPer; ++j) acc[j] = fmaf(w, o[c][j], acc[j]);
          }
        }
      }
    }
  } else {
    for (int pz = lane; pz < NP; pz += 32) {
      const float2 v = __ldcg(md + pz);
      if (v.x > -INFINITY && v.y > 0.f) M = fmaxf(M, v.x);
    }
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
    if (M != -INFINITY) {
      for (int pz = lane; pz < NP; pz += 32) {
        const float2 v = __ldcg(md + pz);
        if (v.x > -INFINITY && v.y > 0.f) L += v.y * fast_exp2(v.x - M);
      }
    }
#pragma unroll
    for (int sh = 16; sh > 0; sh >>= 1) L += __shfl_xor_sync(0xffffffffu, L, sh);
    if (M != -INFINITY) {
      // loads are unconditional (every split's row is in bounds) so the
      // unrolled iterations issue them back to back; empty or invalid splits
      // are dropped by a select, never by multiplying their (unread) values
#pragma unroll 8
      for (int pz = 0; pz < NP; ++pz) {
        const float2 v = __ldcg(md + pz);
        float o[kPer];
        load_partial<HD>(src + static_cast<size_t>(pz) * HD, o);
        const bool valid = v.x > -INFINITY && v.y > 0.f;
        const float w = fast_exp2(v.x - M);
#pragma unroll
        for (int j = 0; j < kPer; ++j) acc[j] = valid ? fmaf(w, o[j], acc[j]) : acc[j];
      }
    }
  }
  M_out = M;
  L_out = L;
}

// Merge the NP split partials of query row r (one warp; lanes own HD/32
// contiguous columns): M = max m_z, L = sum d_z 2^(m_z - M), O = sum o_z
// 2^(m_z - M) / L -- the merge algebra of the reference combine
// (csrc_native/m1_kernel.cpp:862-888), reduced by merge_split_core.
// Partials are read past L1 (__ldcg) so a merge may run in the launch that
// wrote them.
template <typename T, int HD, bool kChunked = true>
__device__ __forceinline__ void merge_split_row(const float* ows, const float* mdws, int r, int NP, int lane,
                                                T* out, float* out_f32, float* lse) {
  constexpr int kPer = HD / 32;
  float acc[kPer], M, L;
  merge_split_core<HD, kChunked>(ows, mdws, r, NP, lane, acc, M, L);
  const float inv = L > 0.f ? 1.f / L : 0.f;
  if (out != nullptr) {
    T* op = out + static_cast<size_t>(r) * HD + lane * kPer;
#pragma unroll
    for (int j = 0; j < kPer; j += 2) *reinterpret_cast<uint32_t*>(op + j) = Elem<T>::pack(acc[j] * inv, acc[j + 1] * inv);
  }
  if (out_f32 != nullptr) {
#pragma unroll
    for (int j = 0; j < kPer; ++j) out_f32[static_cast<size_t>(r) * HD + lane * kPer + j] = acc[j] * inv;
  }
  if (lse != nullptr && lane == 0) lse[r] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
}

// kFp8: e4m3 caches.  Tiles are dequantised in registers (cvt e4m3x2 ->
// f16x2, exact) and both products run in f16; q is converted to f16 once.
// merge_split_row for the exchange: the normalised f32 row and its LSE,
// tagged with step tag, are written to the record slot [rank][r] of every
// rank's exchange buffer (16-byte stores of two tagged words).
template <int HD, bool kChunked = true>
__device__ __forceinline__ void merge_split_row_publish(const float* ows, const float* mdws, int r, int NP,
                                                        int lane, const unsigned long long* bufs, int world,
                                                        int rank, int rows, size_t rec_off, unsigned tag) {
  constexpr int kPer = HD / 32;
  float acc[kPer], M, L;
  merge_split_core<HD, kChunked>(ows, mdws, r, NP, lane, acc, M, L);
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const float lse = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
  for (int dst = 0; dst < world; ++dst) {
    uint64_t* rec = reinterpret_cast<uint64_t*>(bufs[dst] + rec_off) + (static_cast<size_t>(rank) * rows + r) * (HD + 2);
#pragma unroll
    for (int j = 0; j < kPer; j += 2)
      st_words2(rec + lane * kPer + j, cp_word(acc[j] * inv, tag), cp_word(acc[j + 1] * inv, tag));
    if (lane == 0) st_words2(rec + HD, cp_word(lse, tag), cp_word(0.f, tag));
  }
}

// The decode kernel's end-of-unit merges, called out of line: their loads
// and chunk of partial rows then never add to the register pressure of the
// kernel's main loop (the standalone combine kernels inline the same code).
template <typename T, int HD>
__device__ __noinline__ void merge_split_row_call(const float* ows, const float* mdws, int r, int NP, int lane,
                                                  T* out, float* lse) {
  merge_split_row<T, HD>(ows, mdws, r, NP, lane, out, nullptr, lse);
}
template <int HD>
__device__ __noinline__ void merge_split_row_publish_call(const float* ows, const float* mdws, int r, int NP,
                                                          int lane, const unsigned long long* bufs, int world,
                                                          int rank, int rows, size_t rec_off, unsigned tag) {
  merge_split_row_publish<HD>(ows, mdws, r, NP, lane, bufs, world, rank, rows, rec_off, tag);
}

// ------------------------------------------------ context-parallel merge

// One query row (one warp): LSE-merge the world records of row r in rank
// order, once each lane has seen step tag `tag` on its words (bounded wait:
// after kWaitLimitNs from t0 the lane stops waiting, raises the timeout flag
// and merges what it has), and write the output row and its LSE.  A record
// (O, lse) is the partial (o = O, m = lse * log2 e, d = 1).
template <typename T, int HD>
__device__ __forceinline__ void cp_merge_row(const uint64_t* recs, int rows, int r, int world, int lane, T* out,
                                             float* lse, unsigned tag, unsigned long long t0) {
  constexpr int kPer = HD / 32;
  float M = -INFINITY, L = 0.f;
  float acc[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) acc[j] = 0.f;
  bool late = false;
  for (int src = 0; src < world; ++src) {
    const uint64_t* rec = recs + (static_cast<size_t>(src) * rows + r) * (HD + 2);
    uint64_t w[kPer], wl, pad;
    for (;;) {
      bool seen = true;
#pragma unroll
      for (int j = 0; j < kPer; j += 2) {
        ld_words2(rec + lane * kPer + j, w[j], w[j + 1]);
        seen = seen && static_cast<unsigned>(w[j] >> 32) == tag && static_cast<unsigned>(w[j + 1] >> 32) == tag;
      }
      ld_words2(rec + HD, wl, pad);
      if (seen && static_cast<unsigned>(wl >> 32) == tag) break;
      if (late || global_timer_ns() - t0 > kWaitLimitNs) {
        if (!late) raise_flag(MXFA_FLAG_WAIT_TIMEOUT);
        late = true;
        break;
      }
    }
    const float mz = __uint_as_float(static_cast<uint32_t>(wl)) * kLog2e;
    if (!(mz > -INFINITY)) continue;
    const float mn = fmaxf(M, mz);
    const float f1 = fast_exp2(M - mn);
    const float f2 = fast_exp2(mz - mn);
#pragma unroll
    for (int j = 0; j < kPer; ++j) acc[j] = acc[j] * f1 + __uint_as_float(static_cast<uint32_t>(w[j])) * f2;
    L = L * f1 + f2;
    M = mn;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  T* op = out + static_cast<size_t>(r) * HD + lane * kPer;
#pragma unroll
  for (int j = 0; j < kPer; j += 2)
    *reinterpret_cast<uint32_t*>(op + j) = Elem<T>::pack(acc[j] * inv, acc[j + 1] * inv);
  if (lse != nullptr && lane == 0) lse[r] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
}
template <typename T, int HD>
__device__ __noinline__ void cp_merge_row_call(const uint64_t* recs, int rows, int r, int world, int lane, T* out,
                                               float* lse, unsigned tag, unsigned long long t0) {
  cp_merge_row<T, HD>(recs, rows, r, world, lane, out, lse, tag, t0);
}

// e4m3 tiles: token order of the score product.  ldmatrix .m16n16 .trans
// .b8 hands lane (g, t4) the bytes of tokens 4*t4 .. 4*t4+3 for head-dim
// rows g and g+8, so after widening, K-step slots (2*t4, 2*t4+1) of the f16
// P.V product hold tokens (4*t4, 4*t4+1) and slots (2*t4+8, 2*t4+9) tokens
// (4*t4+2, 4*t4+3).  The score product's M rows are loaded in the same
// order (row i is token fp8_tok(i)), so P arrives with its K slots already
// matching V and no register transpose of V is needed.
__device__ __forceinline__ int fp8_tok(int i) { return 4 * ((i & 7) >> 1) + (i & 1) + ((i >> 3) << 1); }

// Two 16x16 byte tiles transposed: lanes 0-15 give the 16 rows of the first,
// lanes 16-31 those of the second.
__device__ __forceinline__ void ldsm_b8_x2_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                 uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m16n16.x2.trans.shared.b8 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T, int HD, int NT, bool kTma, bool kFp8 = false>
__global__ void __launch_bounds__(kDecThreads, DecodeCfg<HD, NT, kFp8>::kCtasPerSm)
    paged_decode_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv) {
  using Cfg = DecodeCfg<HD, NT, kFp8>;
  using MT = std::conditional_t<kFp8, __half, T>;  // tensor-core operand type
  static_assert(DecodeMerge<HD, NT>::kBytes <= Cfg::kRingBytes, "merge scratch must fit the ring");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + Cfg::kRingBytes);
  uint64_t* empty = full + Cfg::kSlots;

  // Programmatic dependent launch: let the next kernel on the stream start
  // placing its blocks as soon as every block of this grid is running (they
  // fill SMs this grid's tail frees), and wait for the previous kernel to
  // finish before touching any input.  Both are no-ops without the launch
  // attribute.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // set-up that reads no input overlaps the predecessor's tail: the slot
  // barriers, and the tensor-map descriptors (kernel parameters) warmed for
  // the producer's first copies
  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kSlots; ++s) {
      mbar_init(&full[s], kTma ? 1 : 32);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
  }
  if (kTma && threadIdx.x == kDecConsumerWarps * 32) {
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // Grid: x = (KV head, row group), y = length rank, z = split.  The hardware
  // dispatches blocks in linear order, so mapping rank y to the y-th longest
  // sequence starts the longest work first (longest-processing-time order),
  // which keeps the tail of ragged batches short.
  const int kvh = blockIdx.x % p.HKV;
  const int rg = blockIdx.x / p.HKV;
  const int z = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int b = blockIdx.y;
  int cached_len = 0;
  bool have_len = false;
  if (p.order != nullptr && p.B > 1 && p.B <= kRankMaxBatch) {
    b = p.order[blockIdx.y];
    if (b < 0 || b >= p.B) {  // not a permutation of the batch: run row y's own sequence
      raise_flag(MXFA_FLAG_BAD_ORDER);
      b = blockIdx.y;
    }
  } else if (p.B > 1 && p.B <= kRankMaxBatch) {
    // Rank every sequence by length (ties by index) and take the one whose
    // rank is this block's y.  Each sequence gets one packed key -- length in
    // the high bits, reversed index in the low 9 -- so keys are unique and a
    // rank is one compare per pair; keys are padded to a multiple of 4 with
    // -1 and read four at a time.  The chosen length comes back with the
    // index so no second global read sits on the start-up path.
    __shared__ int s_seq, s_len;
    int* keys = reinterpret_cast<int*>(ring);  // ring is not in use yet
    int* lens = keys + kRankMaxBatch;
    const int bp = (p.B + 3) & ~3;
    for (int i = threadIdx.x; i < bp; i += blockDim.x) {
      int key = -1;
      if (i < p.B) {
        const int len = p.seqlens[i];
        lens[i] = len;
        key = (min(max(len, 0), (1 << 22) - 1) << 9) | (kRankMaxBatch - 1 - i);
      }
      keys[i] = key;
    }
    __syncthreads();
    const int want = blockIdx.y;
    const int4* keys4 = reinterpret_cast<const int4*>(keys);
    for (int i = threadIdx.x; i < p.B; i += blockDim.x) {
      const int ki = keys[i];
      int rank = 0;
      for (int j4 = 0; j4 < bp / 4; ++j4) {
        const int4 v = keys4[j4];
        rank += (v.x > ki) + (v.y > ki) + (v.z > ki) + (v.w > ki);
      }
      if (rank == want) {
        s_seq = i;
        s_len = lens[i];
      }
    }
    __syncthreads();
    b = s_seq;
    cached_len = s_len;
    have_len = true;
  }

  // split mode (partials written for a combine) whenever a workspace is given;
  // chunk z then covers [z*c_len, (z+1)*c_len) exactly as the reference's split
  const int lo = p.ows != nullptr ? z * p.c_len : 0;
  const int tile0 = (lo / kTileTok) * kTileTok;
  if (!have_len) cached_len = p.seqlens[b];
  const int total_len = cached_len + p.append_len;
  const int hi = p.ows != nullptr ? min(lo + p.c_len, total_len) : total_len;
  const int ntiles = (hi > lo) ? (hi - tile0 + kTileTok - 1) / kTileTok : 0;

  // The producer's first block-table reads go out now, so their latency
  // overlaps the barrier set-up below (only the TMA path uses them).
  int first_rows = 0;
  if (kTma && warp == kDecConsumerWarps) first_rows = tile_slot_row(p, b, tile0, ntiles, lane);

  if (p.k_new != nullptr) {
    // Fused append: this CTA is the only reader of its KV head's positions in
    // [lo, hi), so it writes the appended rows that fall there itself; the
    // proxy fence plus the barrier below order these generic stores before
    // the producer's TMA reads of the same pages.
    const int old_len = total_len - p.append_len;
    const int a_lo = max(lo, old_len), a_hi = min(hi, total_len);
    // positions past the cache's capacity belong to no chunk: report them once
    const int capacity = p.bt != nullptr ? p.BTW * p.PS : p.PS;
    if (threadIdx.x == 0 && z == 0 && rg == 0 && total_len > capacity)
      raise_flag(p.bt != nullptr ? MXFA_FLAG_TABLE_TOO_NARROW : MXFA_FLAG_DENSE_OVERFLOW);
    constexpr int kChunks = Cfg::kRowChunks;
    for (int c = threadIdx.x; c < (a_hi - a_lo) * kChunks; c += blockDim.x) {
      const int pos = a_lo + c / kChunks;
      const int ch = c % kChunks;
      const int page = pos / p.PS;
      int phys = b;
      if (p.bt != nullptr) {
        if (page >= p.BTW) {
          raise_flag(MXFA_FLAG_TABLE_TOO_NARROW);
          continue;
        }
        phys = p.bt[static_cast<size_t>(b) * p.BTW + page];
      } else if (pos >= p.PS) {
        raise_flag(MXFA_FLAG_DENSE_OVERFLOW);
        continue;
      }
      if (phys < 0 || phys >= p.P) {
        raise_flag(MXFA_FLAG_PAGE_OUT_OF_RANGE);
        continue;
      }
      const size_t src =
          ((static_cast<size_t>(b) * p.append_len + (pos - old_len)) * p.HKV + kvh) * Cfg::kRowBytes + ch * 16;
      const size_t dst = ((static_cast<size_t>(phys) * p.PS + pos % p.PS) * p.HKV + kvh) * Cfg::kRowBytes + ch * 16;
      *reinterpret_cast<uint4*>(const_cast<uint8_t*>(static_cast<const uint8_t*>(p.k)) + dst) =
          *reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.k_new) + src);
      *reinterpret_cast<uint4*>(const_cast<uint8_t*>(static_cast<const uint8_t*>(p.v)) + dst) =
          *reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.v_new) + src);
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }

  __syncthreads();  // rank result, appended rows and slot barriers visible to every warp

  // ---------------------------------------------------------------- producer
  if (warp == kDecConsumerWarps) {
    const uint8_t* kc = static_cast<const uint8_t*>(p.k);
    const uint8_t* vc = static_cast<const uint8_t*>(p.v);
    if constexpr (kTma) {
      int abort = 0;
      int issued = 0;  // lane 0: tiles whose copies were started
      for (int base = 0; base < ntiles && !abort; base += 32) {
        // lane j holds the physical slot row of tile base + j (the first 32
        // were resolved before the start-up barrier)
        const int slot_row = base == 0 ? first_rows : tile_slot_row(p, b, tile0, ntiles, base + lane);
        const int n = min(32, ntiles - base);
        for (int j = 0; j < n; ++j) {
          const int row = __shfl_sync(0xffffffffu, slot_row, j);
          if (lane == 0 && !abort) {
            const int tt = base + j;
            const int slot = tt % Cfg::kSlots;
            const int use = tt / Cfg::kSlots;
            if (use > 0 && !mbar_wait(&empty[slot], (use - 1) & 1)) {
              abort = 1;
            } else {
              issued = tt + 1;
              mbar_arrive_expect_tx(&full[slot], 2 * Cfg::kTileBytes);
              uint8_t* kd = ring + slot * Cfg::kSlotBytes;
              uint8_t* vd = kd + Cfg::kTileBytes;
              if constexpr (kFp8) {
                // one box: (128 bytes = one row, head, 16 rows, K|V)
                tma_load_4d(ring + slot * Cfg::kSlotBytes, &tmk, &full[slot], 0, kvh, row, 0);
              } else if (p.kv_map == 5) {
                // one box: (64 columns, head, 16 rows, column block, K|V)
                tma_load_5d(ring + slot * Cfg::kSlotBytes, &tmk, &full[slot], 0, kvh, row, 0, 0);
              } else if (p.kv_map == 4) {
                // one box per tensor: (64 columns, head, 16 rows, column block)
                tma_load_4d(kd, &tmk, &full[slot], 0, kvh, row, 0);
                tma_load_4d(vd, &tmv, &full[slot], 0, kvh, row, 0);
              } else {
#pragma unroll
                for (int db = 0; db < Cfg::kDBlk; ++db) {
                  tma_load_3d(kd + db * Cfg::kBlkBytes, &tmk, &full[slot], db * 64, kvh, row);
                  tma_load_3d(vd + db * Cfg::kBlkBytes, &tmv, &full[slot], db * 64, kvh, row);
                }
              }
            }
          }
          abort = __shfl_sync(0xffffffffu, abort, 0);
          if (abort) break;
        }
      }
      // every copy issued must land before the CTA exits: wait (bounded) for
      // the last phase of each slot used
      if (lane == 0)
        for (int tt = max(issued - Cfg::kSlots, 0); tt < issued; ++tt)
          mbar_wait(&full[tt % Cfg::kSlots], (tt / Cfg::kSlots) & 1);
    } else {
      constexpr int kRowChunks = Cfg::kRowChunks;
      constexpr int kChunks = kTileTok * kRowChunks;  // per tile per tensor (a multiple of 32)
      for (int t = 0; t < ntiles; ++t) {
        const int slot = t % Cfg::kSlots;
        const int use = t / Cfg::kSlots;
        const bool ready = use == 0 || mbar_wait(&empty[slot], (use - 1) & 1);
        if (!__all_sync(0xffffffffu, ready)) break;  // every lane leaves together
        uint8_t* kd = ring + slot * Cfg::kSlotBytes;
        uint8_t* vd = kd + Cfg::kTileBytes;
        const int pos0 = tile0 + t * kTileTok;
        // lane r < 16 resolves row r's element offset once (-1: outside [lo, hi)
        // or not mapped; the slot row is left stale and consumers mask / zero it)
        long long roff = -1;
        if (lane < kTileTok) {
          const int pos = pos0 + lane;
          if (pos >= lo && pos < hi) {
            const int page = pos / p.PS;
            int phys = b;
            bool mapped = true;
            if (p.bt != nullptr) {
              if (page >= p.BTW) {
                raise_flag(MXFA_FLAG_TABLE_TOO_NARROW);
                mapped = false;
              } else {
                phys = p.bt[static_cast<size_t>(b) * p.BTW + page];
              }
            }
            if (mapped && (phys < 0 || phys >= p.P)) {
              raise_flag(MXFA_FLAG_PAGE_OUT_OF_RANGE);
              mapped = false;
            }
            if (mapped)
              roff = ((static_cast<long long>(phys) * p.PS + (pos % p.PS)) * p.HKV + kvh) * Cfg::kRowBytes;
          }
        }
#pragma unroll 4
        for (int c = lane; c < kChunks; c += 32) {
          const int r = c / kRowChunks;
          const int ch = c % kRowChunks;
          const long long off = __shfl_sync(0xffffffffu, roff, r);
          if (off < 0) continue;
          const uint32_t so = (ch >> 3) * Cfg::kBlkBytes + swz128(r, ch & 7);
          cp_async_16(kd + so, kc + off + ch * 16);
          cp_async_16(vd + so, vc + off + ch * 16);
        }
        cp_async_mbar_arrive_noinc(&full[slot]);
      }
      cp_async_wait_all();  // this lane's copies have landed before it exits
    }
    return;
  }

  // ---------------------------------------------------------------- consumers
  const int g = lane >> 2;
  const int t4 = lane & 3;
  const int rows_total = p.Sq * p.GQ;
  const int row_base = rg * 8 * NT;
  const T* qptr = static_cast<const T*>(p.q);

  // Q^T fragments (B operand): thread holds Q[row g][d = kk*16 + 2*t4 + {0,1}, +8]
  uint32_t qf[HD / 16][NT][2];
  int lim[NT][2];  // last visible key position of the two rows this thread owns in each n-tile
  int lim_min = 0x7fffffff;  // the smallest of them over rows that exist
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int row = row_base + nt * 8 + g;
    const T* qr = nullptr;
    if (row < rows_total) {
      const int i = row / p.GQ;
      const int h = kvh * p.GQ + row % p.GQ;
      qr = qptr + (static_cast<size_t>(b * p.Sq + i) * p.HQ + h) * HD;
    }
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      if constexpr (kFp8) {
        // fp8 K fragments come out of ldmatrix with D permuted inside each
        // 16-column step (thread t4 holds columns 4*t4 .. 4*t4+3); q is loaded
        // in the same order and converted to f16
        uint2 v = make_uint2(0u, 0u);
        if (qr) v = *reinterpret_cast<const uint2*>(qr + kk * 16 + 4 * t4);
        qf[kk][nt][0] = to_f16x2<T>(v.x);
        qf[kk][nt][1] = to_f16x2<T>(v.y);
      } else {
        qf[kk][nt][0] = qr ? ld_u32(qr + kk * 16 + 2 * t4) : 0u;
        qf[kk][nt][1] = qr ? ld_u32(qr + kk * 16 + 8 + 2 * t4) : 0u;
      }
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int col_row = row_base + nt * 8 + 2 * t4 + c;
      if (col_row >= rows_total)
        lim[nt][c] = -1;
      else if (p.causal)
        lim[nt][c] = total_len - p.Sq + col_row / p.GQ;
      else
        lim[nt][c] = 0x7fffffff;
      if (col_row < rows_total) lim_min = min(lim_min, lim[nt][c]);
    }
  }

  float m[NT][2], l[NT][2];
  float o[HD / 16][NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m[nt][0] = m[nt][1] = -INFINITY;
    l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
    for (int mi = 0; mi < HD / 16; ++mi)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[mi][nt][e] = 0.f;
  }

  for (int t = warp; t < ntiles; t += kDecConsumerWarps) {
    const int slot = t % Cfg::kSlots;
    if (!mbar_wait(&full[slot], (t / Cfg::kSlots) & 1)) break;
    uint8_t* kd = ring + slot * Cfg::kSlotBytes + (p.kv_swap ? Cfg::kTileBytes : 0);
    uint8_t* vd = ring + slot * Cfg::kSlotBytes + (p.kv_swap ? 0 : Cfg::kTileBytes);
    const int pos0 = tile0 + t * kTileTok;
    const bool partial = (pos0 < lo) || (pos0 + kTileTok > hi);
    if (partial) {
      // rows outside [lo, hi) may hold padding (even NaN): zero their V so p=0 rows add nothing
      for (int c = lane; c < kTileTok * Cfg::kRowChunks; c += 32) {
        const int r = c / Cfg::kRowChunks;
        const int ch = c % Cfg::kRowChunks;
        const int pos = pos0 + r;
        if (pos < lo || pos >= hi)
          *reinterpret_cast<uint4*>(vd + (ch >> 3) * Cfg::kBlkBytes + swz128(r, ch & 7)) =
              make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }
    const uint32_t kbase = smem_u32(kd);
    const uint32_t vbase = smem_u32(vd);

    float s[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    if constexpr (kFp8) {
      // odd K-steps accumulate separately: two independent MMA chains
      float s2[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) s2[nt][0] = s2[nt][1] = s2[nt][2] = s2[nt][3] = 0.f;
      // one ldmatrix.x4 = two 16-column steps x two 8-token halves of fp8 K;
      // each register (4 e4m3 values) becomes the step's low and high f16x2;
      // M row i of the product is token fp8_tok(i)
      const int q8 = lane >> 3;
      const int r = fp8_tok(((q8 & 1) << 3) + (lane & 7));
#pragma unroll
      for (int c2 = 0; c2 < HD / 32; ++c2) {
        uint32_t x[4];
        ldsm_x4(kbase + swz128(r, 2 * c2 + (q8 >> 1)), x[0], x[1], x[2], x[3]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int kk = 2 * c2 + h;
          uint32_t lo0, hi0, lo1, hi1;
          e4m3x4_to_f16x2x2(x[2 * h], lo0, hi0);
          e4m3x4_to_f16x2x2(x[2 * h + 1], lo1, hi1);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            Elem<MT>::mma(h ? s2[nt] : s[nt], lo0, lo1, hi0, hi1, qf[kk][nt][0], qf[kk][nt][1]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[nt][e] += s2[nt][e];
    } else {
      const int q8 = lane >> 3;
      const int r = ((q8 & 1) << 3) + (lane & 7);
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        const int dch = kk * 2 + (q8 >> 1);  // 8-element chunk index along D
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kbase + (dch >> 3) * Cfg::kBlkBytes + swz128(r, dch & 7), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) Elem<MT>::mma(s[nt], a0, a1, a2, a3, qf[kk][nt][0], qf[kk][nt][1]);
      }
    }

    // mask + scale into the log2 domain.  On the e4m3 path (instruction
    // bound), a tile inside [lo, hi) whose last key every existing row sees
    // needs no mask (rows past rows_total have q = 0 and are never read back).
    if (kFp8 && !partial && pos0 + kTileTok - 1 <= lim_min) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[nt][e] *= p.scale_log2;
    } else {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = g + ((e >> 1) << 3);  // M row of the score product
          const int pos = pos0 + (kFp8 ? fp8_tok(row) : row);
          const bool ok = pos >= lo && pos < hi && pos <= lim[nt][e & 1];
          s[nt][e] = ok ? s[nt][e] * p.scale_log2 : -INFINITY;
        }
    }

    // online softmax per query row (a column of S^T)
    float alpha[NT][2];
    bool grew = false;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float mx = fmaxf(s[nt][c], s[nt][c + 2]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        // the e4m3 path keeps its running max until a tile's max exceeds it
        // by more than 2^8 (P then stays below 256, exact in f16 with the
        // hi/lo split), which skips most O rescales
        const float m_cand = fmaxf(m[nt][c], mx);
        const float m_new = (kFp8 && m_cand <= m[nt][c] + 8.f) ? m[nt][c] : m_cand;
        float a = 1.f, p0 = 0.f, p1 = 0.f;
        if (m_new != -INFINITY) {
          a = fast_exp2(m[nt][c] - m_new);
          p0 = fast_exp2(s[nt][c] - m_new);
          p1 = fast_exp2(s[nt][c + 2] - m_new);
        }
        grew |= m_new != m[nt][c];
        alpha[nt][c] = a;
        l[nt][c] = l[nt][c] * a + p0 + p1;
        m[nt][c] = m_new;
        s[nt][c] = p0;
        s[nt][c + 2] = p1;
      }
    // the running max rarely moves after the first tiles: rescale O only when it did
    if (__any_sync(0xffffffffu, grew)) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int mi = 0; mi < HD / 16; ++mi) {
          o[mi][nt][0] *= alpha[nt][0];
          o[mi][nt][1] *= alpha[nt][1];
          o[mi][nt][2] *= alpha[nt][0];
          o[mi][nt][3] *= alpha[nt][1];
        }
    }

    // P (tok x rows) -> B fragments of the PV product.  P is split into a
    // rounded high part and the rounded remainder (p = hi + lo to ~16
    // significant bits) and both are multiplied with V, so the product keeps
    // fp32-level accuracy even when V carries large outliers; the extra
    // tensor-core work is free on this memory-bound path.  The e4m3 path
    // (instruction bound) multiplies the rounded P only: its f16 rounding
    // (2^-11 relative) lies far below the e4m3 quantisation of the cache
    // (2^-4 relative).
    uint32_t pb[NT][2], pl[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float a = s[nt][2 * hh], c = s[nt][2 * hh + 1];
        const uint32_t hi = Elem<MT>::pack(a, c);
        pb[nt][hh] = movmatrix_trans(hi);
        if constexpr (!kFp8) {
          const float2 hf = Elem<MT>::unpack(hi);
          pl[nt][hh] = movmatrix_trans(Elem<MT>::pack(a - hf.x, c - hf.y));
        }
      }
    if constexpr (kFp8) {
      // fp8 V through the transposing 8-bit ldmatrix: for head-dim step mi,
      // lane (g, t4) gets V[tokens 4*t4..4*t4+3][d = 16*mi + g] and [.. + 8];
      // widened, these are the A fragment of V^T with the token order of P
      // (see fp8_tok), so the accumulator keeps the natural D order
      const int vrow = lane & 15;  // token row this lane addresses
#pragma unroll
      for (int mi = 0; mi < HD / 16; mi += 2) {
        uint32_t y0, y1, y2, y3;
        ldsm_b8_x2_trans(vbase + swz128(vrow, mi + (lane >> 4)), y0, y1, y2, y3);
        const uint32_t yy[2][2] = {{y0, y1}, {y2, y3}};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t a0, a2, a1, a3;
          e4m3x4_to_f16x2x2(yy[h][0], a0, a2);  // d = 16*(mi+h) + g: token slots 2*t4.. and 2*t4+8..
          e4m3x4_to_f16x2x2(yy[h][1], a1, a3);  // d = 16*(mi+h) + g + 8
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) Elem<MT>::mma(o[mi + h][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
        }
      }
    } else {
      const int q8 = lane >> 3;
      const int r = ((q8 >> 1) << 3) + (lane & 7);
#pragma unroll
      for (int mi = 0; mi < HD / 16; ++mi) {
        const int dch = mi * 2 + (q8 & 1);
        uint32_t a0, a1, a2, a3;
        ldsm_x4_trans(vbase + (dch >> 3) * Cfg::kBlkBytes + swz128(r, dch & 7), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          Elem<MT>::mma(o[mi][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
          Elem<MT>::mma(o[mi][nt], a0, a1, a2, a3, pl[nt][0], pl[nt][1]);
        }
      }
    }
    __syncwarp();
    if (partial) fence_proxy_async_smem();  // generic zero-stores before the next TMA write
    if (lane == 0) mbar_arrive(&empty[slot]);
  }

  // row sums: reduce over the 8 token groups
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      l[nt][c] += __shfl_xor_sync(0xffffffffu, l[nt][c], 4);
      l[nt][c] += __shfl_xor_sync(0xffffffffu, l[nt][c], 8);
      l[nt][c] += __shfl_xor_sync(0xffffffffu, l[nt][c], 16);
    }

  // ---------------------------------------------------- merge the 4 warps
  using Mg = DecodeMerge<HD, NT>;
  named_barrier_sync(1, kDecConsumerWarps * 32);  // every consumer finished reading the ring
  float* om = reinterpret_cast<float*>(ring);
  float* mm = reinterpret_cast<float*>(ring + Mg::kOBytes);
  float* lm = mm + kDecConsumerWarps * Mg::kCols;
#pragma unroll
  for (int mi = 0; mi < HD / 16; ++mi)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = nt * 8 + 2 * t4 + (e & 1);
        const int d = mi * 16 + g + ((e >> 1) << 3);
        om[(warp * Mg::kCols + col) * Mg::kStride + d] = kFp8 ? o[mi][nt][e] * p.v_scale : o[mi][nt][e];
      }
  if (g == 0) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int col = nt * 8 + 2 * t4 + c;
        mm[warp * Mg::kCols + col] = m[nt][c];
        lm[warp * Mg::kCols + col] = l[nt][c];
      }
  }
  named_barrier_sync(1, kDecConsumerWarps * 32);

  const int tid = threadIdx.x;
  constexpr int kQuads = HD / 4;
  for (int idx = tid; idx < Mg::kCols * kQuads; idx += kDecConsumerWarps * 32) {
    const int col = idx / kQuads;
    const int d4 = (idx % kQuads) * 4;
    const int rr = row_base + col;
    if (rr >= rows_total) continue;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecConsumerWarps; ++w) M = fmaxf(M, mm[w * Mg::kCols + col]);
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kDecConsumerWarps; ++w) {
        const float f = fast_exp2(mm[w * Mg::kCols + col] - M);
        L += lm[w * Mg::kCols + col] * f;
        const float4 ow = *reinterpret_cast<const float4*>(&om[(w * Mg::kCols + col) * Mg::kStride + d4]);
        acc.x += ow.x * f;
        acc.y += ow.y * f;
        acc.z += ow.z * f;
        acc.w += ow.w * f;
      }
    }
    const int i = rr / p.GQ;
    const int h = kvh * p.GQ + rr % p.GQ;
    const size_t R = static_cast<size_t>(b * p.Sq + i) * p.HQ + h;
    if (p.ows != nullptr) {
      *reinterpret_cast<float4*>(p.ows + (R * p.NP + z) * HD + d4) = acc;
      if (d4 == 0) {
        p.mdws[(R * p.NP + z) * 2] = M;
        p.mdws[(R * p.NP + z) * 2 + 1] = L;
      }
    } else {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      T* op = static_cast<T*>(p.out) + R * HD + d4;
      uint2 packed;
      packed.x = Elem<T>::pack(acc.x * inv, acc.y * inv);
      packed.y = Elem<T>::pack(acc.z * inv, acc.w * inv);
      *reinterpret_cast<uint2*>(op) = packed;
      if (d4 == 0 && p.lse != nullptr) p.lse[R] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
    }
  }

  if (p.counters != nullptr && p.ows != nullptr) {
    // Single-launch split: publish this chunk's partials, count it, and let
    // the last chunk of the unit merge all of them.
    __shared__ int s_last;
    __threadfence();
    named_barrier_sync(1, kDecConsumerWarps * 32);
    unsigned* counter = p.counters + static_cast<size_t>(b) * gridDim.x + blockIdx.x;
    if (tid == 0) s_last = atomicAdd(counter, 1u) == gridDim.z - 1;
    named_barrier_sync(1, kDecConsumerWarps * 32);
    if (s_last) {
      __threadfence();
      const int rows_all = p.B * p.Sq * p.HQ;
      const CpLayout lay = cp_layout(p.cp_world, rows_all, HD);
      const unsigned epoch =
          p.cp_bufs != nullptr ? *reinterpret_cast<const volatile unsigned*>(p.cp_bufs[p.cp_rank]) : 0u;
      const unsigned tag = epoch + 1u;
      const size_t rec_off = lay.records + (epoch & 1u) * lay.record_half;
      for (int col = warp; col < Mg::kCols; col += kDecConsumerWarps) {
        const int rr = row_base + col;
        if (rr >= rows_total) break;
        const int i = rr / p.GQ;
        const int h = kvh * p.GQ + rr % p.GQ;
        const int R = (b * p.Sq + i) * p.HQ + h;
        if constexpr (kFp8) {
          // the e4m3 kernel runs at its register cap: the loop form, inline
          if (p.cp_bufs != nullptr)
            merge_split_row_publish<HD, false>(p.ows, p.mdws, R, p.NP, lane, p.cp_bufs, p.cp_world, p.cp_rank,
                                               rows_all, rec_off, tag);
          else
            merge_split_row<T, HD, false>(p.ows, p.mdws, R, p.NP, lane, static_cast<T*>(p.out), nullptr, p.lse);
        } else if (p.cp_bufs != nullptr) {
          merge_split_row_publish_call<HD>(p.ows, p.mdws, R, p.NP, lane, p.cp_bufs, p.cp_world, p.cp_rank, rows_all,
                                           rec_off, tag);
        } else {
          merge_split_row_call<T, HD>(p.ows, p.mdws, R, p.NP, lane, static_cast<T*>(p.out), p.lse);
        }
      }
      if constexpr (!kFp8) {
        if (p.cp_bufs != nullptr && p.cp_merge) {
          // Merge this unit's rows as soon as every rank's words for them carry
          // this step's tag (each warp reads back the rows it published, so the
          // local record needs no ordering beyond program order).
          unsigned char* local = reinterpret_cast<unsigned char*>(p.cp_bufs[p.cp_rank]);
          const uint64_t* recs = reinterpret_cast<const uint64_t*>(local + rec_off);
          const unsigned long long t0 = global_timer_ns();
          for (int col = warp; col < Mg::kCols; col += kDecConsumerWarps) {
            const int rr = row_base + col;
            if (rr >= rows_total) break;
            const int h = kvh * p.GQ + rr % p.GQ;
            const int R = (b * p.Sq + rr / p.GQ) * p.HQ + h;
            cp_merge_row_call<T, HD>(recs, rows_all, R, p.cp_world, lane, static_cast<T*>(p.out), p.lse, tag, t0);
          }
          __syncwarp();  // lanes leave their per-word waits at different times
          named_barrier_sync(1, kDecConsumerWarps * 32);
          if (tid == 0) {
            __threadfence();
            unsigned* hdr = reinterpret_cast<unsigned*>(local);
            if (atomicAdd(hdr + 1, 1u) == static_cast<unsigned>(p.B * gridDim.x) - 1u) {  // every unit merged
              hdr[1] = 0u;
              *reinterpret_cast<volatile unsigned*>(hdr) = epoch + 1u;
            }
          }
        }
      }
      if (tid == 0) *counter = 0u;  // ready for the next launch on this stream
    }
  }
}

// --------------------------------------------------------------- combine

// One warp per query row; lanes own D/32 contiguous columns.  Partial p of
// row r: o at ows[(r*NP + p)*D], (m, d) at mdws[(r*NP + p)*2].  PACKED_LSE
// reads per-rank (O, LSE) rows instead: packed[(p*rows + r)*(D+1)] holds the
// normalised O followed by the natural-log LSE.
// With kPackedOut the f32 result is written packed per row, O then LSE
// ([rows, D+1]): the record one rank contributes to a context-split merge.
template <typename T, int HD, bool kPackedLse, bool kPackedOut = false>
__global__ void __launch_bounds__(128) split_combine_kernel(const float* __restrict__ ows,
                                                            const float* __restrict__ mdws,
                                                            T* __restrict__ out, float* __restrict__ out_f32,
                                                            float* __restrict__ lse, int rows, int NP) {
  constexpr int kPer = HD / 32;
  const int r = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  if constexpr (!kPackedLse && !kPackedOut) {
    merge_split_row<T, HD>(ows, mdws, r, NP, lane, out, out_f32, lse);
    return;
  }
  float M = -INFINITY, L = 0.f;
  float acc[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) acc[j] = 0.f;
  for (int pz = 0; pz < NP; ++pz) {
    float mz, dz;
    const float* src;
    if constexpr (kPackedLse) {
      src = ows + (static_cast<size_t>(pz) * rows + r) * (HD + 1);
      const float lz = src[HD];
      mz = lz * kLog2e;  // (O, lse) == (o = O, m = lse*log2e, d = 1)
      dz = 1.f;
    } else {
      const size_t pi = static_cast<size_t>(r) * NP + pz;
      mz = mdws[pi * 2];
      dz = mdws[pi * 2 + 1];
      src = ows + pi * HD;
    }
    if (!(mz > -INFINITY) || !(dz > 0.f)) continue;
    const float mn = fmaxf(M, mz);
    const float f1 = fast_exp2(M - mn);
    const float f2 = fast_exp2(mz - mn);
    float vals[kPer];
    if constexpr (kPer == 4 && !kPackedLse) {
      const float4 v4 = *reinterpret_cast<const float4*>(src + lane * 4);
      vals[0] = v4.x; vals[1] = v4.y; vals[2] = v4.z; vals[3] = v4.w;
    } else {
#pragma unroll
      for (int j = 0; j < kPer; ++j) vals[j] = src[lane * kPer + j];
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) acc[j] = acc[j] * f1 + vals[j] * f2;
    L = L * f1 + dz * f2;
    M = mn;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  if (out != nullptr) {
    T* op = out + static_cast<size_t>(r) * HD + lane * kPer;
#pragma unroll
    for (int j = 0; j < kPer; j += 2) *reinterpret_cast<uint32_t*>(op + j) = Elem<T>::pack(acc[j] * inv, acc[j + 1] * inv);
  }
  if constexpr (kPackedOut) {
    float* row = out_f32 + static_cast<size_t>(r) * (HD + 1);
#pragma unroll
    for (int j = 0; j < kPer; ++j) row[lane * kPer + j] = acc[j] * inv;
    if (lane == 0) row[HD] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
  } else {
    if (out_f32 != nullptr) {
#pragma unroll
      for (int j = 0; j < kPer; ++j) out_f32[static_cast<size_t>(r) * HD + lane * kPer + j] = acc[j] * inv;
    }
    if (lse != nullptr && lane == 0) lse[r] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
  }
}

// ------------------------------------- context-parallel merge, second launch

// The merge as its own kernel, for grids whose units do not all fit on the
// GPU at once (the decode kernel merges in place otherwise).  One warp per
// query row on each rank merges the row's records once every rank's words
// carry this step's tag (bounded wait).  The last block to finish advances
// the epoch.
template <typename T, int HD>
__global__ void __launch_bounds__(128) cp_merge_kernel(unsigned char* buf, T* __restrict__ out,
                                                       float* __restrict__ lse, int rows, int world) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int r = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  unsigned* hdr = reinterpret_cast<unsigned*>(buf);
  const unsigned epoch = *reinterpret_cast<volatile unsigned*>(hdr);
  const CpLayout lay = cp_layout(world, rows, HD);
  if (r < rows)
    cp_merge_row<T, HD>(reinterpret_cast<const uint64_t*>(buf + lay.records + (epoch & 1u) * lay.record_half), rows,
                        r, world, lane, out, lse, epoch + 1u, global_timer_ns());
  __syncwarp();  // lanes leave their per-word waits at different times
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(hdr + 1, 1u) == gridDim.x - 1) {
      hdr[1] = 0u;
      *reinterpret_cast<volatile unsigned*>(hdr) = epoch + 1u;
    }
  }
}

// ---------------------------------------------------------------- append

struct AppendParams {
  const uint8_t* k_new;  // [B, Sk, HKV, D]
  const uint8_t* v_new;
  uint8_t* k_cache;
  uint8_t* v_cache;
  const int* bt;         // nullptr: dense cache [B, PS, HKV, D]
  const int* seqlens;
  int B, Sk, HKV, row_bytes, PS, BTW, P;
};

// One thread per 16-byte chunk of an appended row: bit-exact placement of
// token i of sequence b at logical position seqlens[b] + i.
__global__ void __launch_bounds__(256) kv_append_kernel(const AppendParams p) {
  const int chunks = p.row_bytes / 16;
  const long long total = static_cast<long long>(p.B) * p.Sk * p.HKV * chunks;
  for (long long idx = blockIdx.x * 256LL + threadIdx.x; idx < total; idx += 256LL * gridDim.x) {
    const int c = static_cast<int>(idx % chunks);
    long long rest = idx / chunks;
    const int h = static_cast<int>(rest % p.HKV);
    rest /= p.HKV;
    const int i = static_cast<int>(rest % p.Sk);
    const int b = static_cast<int>(rest / p.Sk);
    const int pos = p.seqlens[b] + i;
    int phys = b;
    int slot = pos;
    if (p.bt != nullptr) {
      const int page = pos / p.PS;
      if (pos < 0 || page >= p.BTW) {
        raise_flag(MXFA_FLAG_TABLE_TOO_NARROW);
        continue;
      }
      phys = p.bt[static_cast<size_t>(b) * p.BTW + page];
      slot = pos % p.PS;
      if (phys < 0 || phys >= p.P) {
        raise_flag(MXFA_FLAG_PAGE_OUT_OF_RANGE);
        continue;
      }
    } else if (pos < 0 || pos >= p.PS) {
      raise_flag(MXFA_FLAG_DENSE_OVERFLOW);
      continue;
    }
    const size_t src = ((static_cast<size_t>(b) * p.Sk + i) * p.HKV + h) * p.row_bytes + c * 16;
    const size_t dst = ((static_cast<size_t>(phys) * p.PS + slot) * p.HKV + h) * p.row_bytes + c * 16;
    *reinterpret_cast<uint4*>(p.k_cache + dst) = *reinterpret_cast<const uint4*>(p.k_new + src);
    *reinterpret_cast<uint4*>(p.v_cache + dst) = *reinterpret_cast<const uint4*>(p.v_new + src);
  }
}

// Longest-first order of a batch (ties by index), the permutation the decode
// kernel otherwise derives in every CTA: one block, thread i ranks sequence i
// against all others with the same packed key (length in the high bits,
// reversed index in the low 9) and writes order[rank] = i.
__global__ void __launch_bounds__(kRankMaxBatch) length_order_kernel(const int* __restrict__ seqlens, int B,
                                                                     int* __restrict__ order) {
  __shared__ int keys[kRankMaxBatch];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int i = threadIdx.x;
  int key = -1;
  if (i < B) key = (min(max(seqlens[i], 0), (1 << 22) - 1) << 9) | (kRankMaxBatch - 1 - i);
  keys[i] = key;
  __syncthreads();
  if (i < B) {
    int rank = 0;
    for (int j = 0; j < B; ++j) rank += keys[j] > key;
    order[rank] = i;
  }
}

__global__ void seqlens_add_kernel(void* seqlens, int is_int64, int B, int delta) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  if (is_int64)
    static_cast<long long*>(seqlens)[b] += delta;
  else
    static_cast<int*>(seqlens)[b] += delta;
}

}  // namespace mxfa
