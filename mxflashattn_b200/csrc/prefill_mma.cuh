// prefill_mma.cuh -- causal / non-causal varlen attention forward on the
// m16n8k16 tensor-core path (register-resident online softmax).
//
// CTA = 4 warps = 64 query rows of one head of one sequence; K/V stream in
// 64-key tiles, double-buffered with cp.async into 128-byte-swizzled shared
// memory.  Causal masking is bottom-right aligned like the reference
// (mxflashattn/reference.py:31-35): query i of a sequence with Lq queries and
// Lk keys sees keys j <= i + Lk - Lq; a row that sees no key outputs 0
// (reference.py:37-38).  Query tiles are scheduled heaviest-first.
#pragma once

#include "common.cuh"

namespace mxfa {

struct PrefillParams {
  const void* q;      // [Tq, HQ, D]
  const void* k;      // [Tk, HKV, D]
  const void* v;
  const int* cu_q;    // [B+1] or nullptr (uniform lengths Sq / Sk)
  const int* cu_k;
  void* out;          // [Tq, HQ, D]
  float* lse;         // optional [Tq, HQ]
  int B, Sq, Sk, HQ, HKV, GQ;
  int causal;
  float scale_log2;
};

constexpr int kPfRows = 64;   // query rows per CTA
constexpr int kPfKeys = 64;   // keys per tile
constexpr int kPfThreads = 128;

template <int HD>
struct PrefillCfg {
  static constexpr int kDBlk = HD / 64;
  static constexpr int kTileBytes = 64 * HD * 2;   // 64 rows x HD (Q, K or V)
  static constexpr int kBlkBytes = 64 * 128;       // one 64-column block of a tile
  static constexpr int kSmemBytes = 5 * kTileBytes + 1024;  // Q + 2x(K,V)
};

template <int HD>
__device__ __forceinline__ void pf_load_tile(uint8_t* dst, const uint8_t* base, int row0, int rows_valid,
                                             int heads, int head, int tid) {
  // 64 rows x HD elements, row r of the tile = token row0 + r, 16-byte chunks
  constexpr int kChunks = 64 * (HD / 8);
  for (int c = tid; c < kChunks; c += kPfThreads) {
    const int r = c / (HD / 8);
    const int ch = c % (HD / 8);
    const bool ok = r < rows_valid;
    const size_t off = ((static_cast<size_t>(row0 + (ok ? r : 0)) * heads + head) * HD + ch * 8) * 2;
    cp_async_16_zfill(dst + (ch >> 3) * PrefillCfg<HD>::kBlkBytes + swz128(r, ch & 7), base + off, ok);
  }
}

template <typename T, int HD>
__global__ void __launch_bounds__(kPfThreads, 2) prefill_mma_kernel(const PrefillParams p) {
  using Cfg = PrefillCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = sm;
  uint8_t* ks[2] = {sm + Cfg::kTileBytes, sm + 3 * Cfg::kTileBytes};
  uint8_t* vs[2] = {sm + 2 * Cfg::kTileBytes, sm + 4 * Cfg::kTileBytes};

  const int b = blockIdx.z;
  const int h = blockIdx.y;
  const int hk = h / p.GQ;
  int q_start, q_len, k_start, k_len;
  if (p.cu_q != nullptr) {
    q_start = p.cu_q[b];
    q_len = p.cu_q[b + 1] - q_start;
    k_start = p.cu_k[b];
    k_len = p.cu_k[b + 1] - k_start;
  } else {
    q_start = b * p.Sq;
    q_len = p.Sq;
    k_start = b * p.Sk;
    k_len = p.Sk;
  }
  const int qt = gridDim.x - 1 - blockIdx.x;  // heaviest (latest, causal) tiles first
  const int q0 = qt * kPfRows;
  if (q0 >= q_len) return;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int shift = k_len - q_len;  // bottom-right causal alignment

  int k_end = k_len;
  if (p.causal) k_end = min(k_len, q0 + kPfRows - 1 + shift + 1);
  const int nkt = k_end > 0 ? (k_end + kPfKeys - 1) / kPfKeys : 0;

  const uint8_t* qg = static_cast<const uint8_t*>(p.q);
  const uint8_t* kg = static_cast<const uint8_t*>(p.k);
  const uint8_t* vg = static_cast<const uint8_t*>(p.v);

  pf_load_tile<HD>(qs, qg, q_start + q0, q_len - q0, p.HQ, h, tid);
  cp_async_commit();
  if (nkt > 0) {
    pf_load_tile<HD>(ks[0], kg, k_start, k_len, p.HKV, hk, tid);
    pf_load_tile<HD>(vs[0], vg, k_start, k_len, p.HKV, hk, tid);
  }
  cp_async_commit();

  float o[HD / 8][4];
#pragma unroll
  for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  uint32_t qa[HD / 16][4];
  const int row_g[2] = {q0 + warp * 16 + g, q0 + warp * 16 + g + 8};  // query index within sequence

  for (int j = 0; j < nkt; ++j) {
    if (j + 1 < nkt) {
      const int kr = (j + 1) * kPfKeys;
      pf_load_tile<HD>(ks[(j + 1) & 1], kg, k_start + kr, k_len - kr, p.HKV, hk, tid);
      pf_load_tile<HD>(vs[(j + 1) & 1], vg, k_start + kr, k_len - kr, p.HKV, hk, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
      const int q8 = lane >> 3;
      const int r = warp * 16 + ((q8 & 1) << 3) + (lane & 7);
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        const int dch = kk * 2 + (q8 >> 1);
        ldsm_x4(smem_u32(qs) + (dch >> 3) * Cfg::kBlkBytes + swz128(r, dch & 7), qa[kk][0], qa[kk][1],
                qa[kk][2], qa[kk][3]);
      }
    }
    const uint32_t kb = smem_u32(ks[j & 1]);
    const uint32_t vb = smem_u32(vs[j & 1]);

    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
    {
      const int q8 = lane >> 3;
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        const int r = (n + (q8 >> 1)) * 8 + (lane & 7);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const int dch = kk * 2 + (q8 & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kb + (dch >> 3) * Cfg::kBlkBytes + swz128(r, dch & 7), b0, b1, b2, b3);
          Elem<T>::mma(s[n], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
          Elem<T>::mma(s[n + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
        }
      }
    }
    // mask + scale
    const int key0 = j * kPfKeys;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + n * 8 + 2 * t4 + (e & 1);
        const int qi = row_g[e >> 1];
        const bool ok = key < k_len && (!p.causal || key <= qi + shift);
        s[n][e] = ok ? s[n][e] * p.scale_log2 : -INFINITY;
      }
    // online softmax (rows g and g+8 of this warp; a row spans the 4 lanes of a quad)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) mx = fmaxf(mx, fmaxf(s[n][2 * hr], s[n][2 * hr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m[hr], mx);
      float alpha = 1.f, rs = 0.f;
      if (m_new != -INFINITY) {
        alpha = fast_exp2(m[hr] - m_new);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          s[n][2 * hr] = fast_exp2(s[n][2 * hr] - m_new);
          s[n][2 * hr + 1] = fast_exp2(s[n][2 * hr + 1] - m_new);
          rs += s[n][2 * hr] + s[n][2 * hr + 1];
        }
      } else {
#pragma unroll
        for (int n = 0; n < 8; ++n) s[n][2 * hr] = s[n][2 * hr + 1] = 0.f;
      }
      l[hr] = l[hr] * alpha + rs;
      m[hr] = m_new;
#pragma unroll
      for (int dn = 0; dn < HD / 8; ++dn) {
        o[dn][2 * hr] *= alpha;
        o[dn][2 * hr + 1] *= alpha;
      }
    }
    // O += P V
#pragma unroll
    for (int kk2 = 0; kk2 < 4; ++kk2) {
      const uint32_t a0 = Elem<T>::pack(s[2 * kk2][0], s[2 * kk2][1]);
      const uint32_t a1 = Elem<T>::pack(s[2 * kk2][2], s[2 * kk2][3]);
      const uint32_t a2 = Elem<T>::pack(s[2 * kk2 + 1][0], s[2 * kk2 + 1][1]);
      const uint32_t a3 = Elem<T>::pack(s[2 * kk2 + 1][2], s[2 * kk2 + 1][3]);
      const int q8 = lane >> 3;
      const int r = kk2 * 16 + ((q8 & 1) << 3) + (lane & 7);
#pragma unroll
      for (int dn = 0; dn < HD / 8; dn += 2) {
        const int dch = dn + (q8 >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_trans(vb + (dch >> 3) * Cfg::kBlkBytes + swz128(r, dch & 7), b0, b1, b2, b3);
        Elem<T>::mma(o[dn], a0, a1, a2, a3, b0, b1);
        Elem<T>::mma(o[dn + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // this stage is overwritten by the load issued next iteration
  }

  cp_async_wait<0>();  // no copy may still target shared memory when the CTA retires

  // finalize
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    l[hr] += __shfl_xor_sync(0xffffffffu, l[hr], 1);
    l[hr] += __shfl_xor_sync(0xffffffffu, l[hr], 2);
  }
  T* outp = static_cast<T*>(p.out);
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int qi = row_g[hr];
    if (qi >= q_len) continue;
    const float inv = l[hr] > 0.f ? 1.f / l[hr] : 0.f;
    T* orow = outp + (static_cast<size_t>(q_start + qi) * p.HQ + h) * HD;
#pragma unroll
    for (int dn = 0; dn < HD / 8; ++dn)
      *reinterpret_cast<uint32_t*>(orow + dn * 8 + 2 * t4) =
          Elem<T>::pack(o[dn][2 * hr] * inv, o[dn][2 * hr + 1] * inv);
    if (p.lse != nullptr && t4 == 0)
      p.lse[static_cast<size_t>(q_start + qi) * p.HQ + h] =
          l[hr] > 0.f ? (m[hr] + log2f(l[hr])) * kLn2 : -INFINITY;
  }
}

}  // namespace mxfa
