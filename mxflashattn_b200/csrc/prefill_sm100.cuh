// prefill_sm100.cuh -- attention forward on the 5th-generation tensor cores
// (tcgen05 MMA, accumulators in tensor memory, operands staged by TMA).
//
// CTA = one 128-row query tile of one head; 8 warps, specialised:
//   warp 0   : TMA producer -- Q once, then K and V tiles (128 keys) into a
//              two-stage ring, each stage guarded by full/empty mbarriers
//   warp 1   : allocates tensor memory and issues every tcgen05.mma from one
//              thread:  S_j = Q K_j^T  (M=128, N=128, K=D; both K-major)
//                       O  += P_j V_j  (M=128, N=D,  K=128; V MN-major)
//              committing each group to an mbarrier
//   warps 4-7: softmax, one thread per query row (tensor-memory lane = row):
//              read S_j with tcgen05.ld, mask, keep an online max in the log2
//              domain, write P_j (bf16/fp16) into tensor memory for the P.V
//              product (A operand read from TMEM), rescale O in tensor memory
//              only when a row max grows by more than 2^8 (rare after the
//              first tiles), and finally normalise O and store it.
// Tensor memory: S double buffer (2 x 128 fp32 columns) | O (D columns) |
// P double buffer (2 x 64 columns, two 16-bit values per column).
// S_{j+1} is issued before P_j is ready, so the tensor pipe computes the next
// scores while the softmax warps work on the current ones.
//
// Semantics follow mxflashattn/reference.py:8-85: GQA head h reads KV head
// h / (HQ/HKV); causal masking is bottom-right aligned; a row that sees no
// key outputs 0 (LSE -inf).  Every wait is bounded; on a timeout the CTA
// records MXFA_FLAG_WAIT_TIMEOUT, stops, and still frees its tensor memory.
#pragma once

#include <type_traits>

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

// ------------------------------------------------------------ tcgen05 helpers

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16 or fp16 in, fp32 accumulate)
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]: A (M rows = lanes, K packed two 16-bit values per column) read
// straight from tensor memory, so the softmax output never travels through shared memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

#define MXFA_R32(x)                                                                                             \
  "=r"(x[0]), "=r"(x[1]), "=r"(x[2]), "=r"(x[3]), "=r"(x[4]), "=r"(x[5]), "=r"(x[6]), "=r"(x[7]), "=r"(x[8]),   \
      "=r"(x[9]), "=r"(x[10]), "=r"(x[11]), "=r"(x[12]), "=r"(x[13]), "=r"(x[14]), "=r"(x[15]), "=r"(x[16]),    \
      "=r"(x[17]), "=r"(x[18]), "=r"(x[19]), "=r"(x[20]), "=r"(x[21]), "=r"(x[22]), "=r"(x[23]), "=r"(x[24]),   \
      "=r"(x[25]), "=r"(x[26]), "=r"(x[27]), "=r"(x[28]), "=r"(x[29]), "=r"(x[30]), "=r"(x[31])
#define MXFA_W32(x)                                                                                             \
  "r"(x[0]), "r"(x[1]), "r"(x[2]), "r"(x[3]), "r"(x[4]), "r"(x[5]), "r"(x[6]), "r"(x[7]), "r"(x[8]), "r"(x[9]), \
      "r"(x[10]), "r"(x[11]), "r"(x[12]), "r"(x[13]), "r"(x[14]), "r"(x[15]), "r"(x[16]), "r"(x[17]),           \
      "r"(x[18]), "r"(x[19]), "r"(x[20]), "r"(x[21]), "r"(x[22]), "r"(x[23]), "r"(x[24]), "r"(x[25]),           \
      "r"(x[26]), "r"(x[27]), "r"(x[28]), "r"(x[29]), "r"(x[30]), "r"(x[31])

// This warp's 32 lanes x 32 consecutive 32-bit columns starting at `taddr`;
// thread t receives lane (warp%4)*32 + t.  The wait is inside the same asm
// statement, so the registers are valid when it returns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : MXFA_R32(r)
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      MXFA_W32(r)
      : "memory");
}

// Shared-memory matrix descriptor: 128-byte swizzle, descriptor version 1.
//   K-major operand (rows of 64 elements = 128 B): lbo = 16 B (unused), sbo = 1024 B (8-row group stride)
//   MN-major operand (128-B rows run along N): lbo = stride between 64-wide N blocks,
//                                              sbo = 1024 B (8-row group stride along K)
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: fp32 accumulate, A K-major, B K- or MN-major.
template <typename T>
__host__ __device__ constexpr uint32_t umma_idesc(int M, int N, bool b_mn_major) {
  return (1u << 4) | ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 7) |
         ((std::is_same<T, __nv_bfloat16>::value ? 1u : 0u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// --------------------------------------------------------------- layout

constexpr int kTcRows = 128;   // query rows per CTA (MMA M)
constexpr int kTcKeys = 128;   // keys per tile (MMA N of S, K of P.V)
constexpr int kTcThreads = 256;
constexpr int kTcSoftmaxWarps = 4;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O when a row max grows by > 2^8

template <int HD>
struct TcCfg {
  static constexpr int kDBlk = HD / 64;
  static constexpr int kStages = 3;
  static constexpr int kBlk = 128 * 128;               // one 64-column block of a 128-row tile
  static constexpr int kTile = kDBlk * kBlk;           // Q, K or V tile bytes
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kTile;
  static constexpr int kV = kK + kStages * kTile;
  static constexpr int kBar = kV + kStages * kTile;
  static constexpr int kNumBars = 1 + 4 * kStages + 8;
  static constexpr int kSmemBytes = kBar + kNumBars * 8 + 16 + 1024;
  static constexpr uint32_t kTmemCols = 512;            // S0 | S1 | O | P0 P1
  static constexpr uint32_t kTmemO = 256;
  static constexpr uint32_t kTmemP = 384;               // two 64-column P buffers (128 keys, 2 per column)
};

template <int kStages>
struct TcBars {
  uint64_t q_full, k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
  uint64_t s_full[2], s_empty[2], p_full[2], pv_done[2];
};

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      raise_flag(MXFA_FLAG_WAIT_TIMEOUT);
      *abort = 1;
      return false;
    }
  }
}

template <typename T, int HD>
__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_tc_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tmq,
                      const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv) {
  using Cfg = TcCfg<HD>;
  constexpr int NS = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  TcBars<NS>* bars = reinterpret_cast<TcBars<NS>*>(sm + Cfg::kBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Cfg::kBar + Cfg::kNumBars * 8);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
  const int q0 = qt * kTcRows;
  if (q0 >= q_len) return;
  const int shift = k_len - q_len;
  const int last_row = min(q0 + kTcRows, q_len) - 1;
  const int k_end = p.causal ? min(k_len, last_row + shift + 1) : k_len;
  const int nkt = k_end > 0 ? (k_end + kTcKeys - 1) / kTcKeys : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  T* outp = static_cast<T*>(p.out);
  if (nkt == 0) {  // every row of this tile sees no key: output 0, LSE -inf
    if (warp >= 4) {
      const int r = (warp - 4) * 32 + lane;
      if (q0 + r < q_len) {
        T* orow = outp + (static_cast<size_t>(q_start + q0 + r) * p.HQ + h) * HD;
        for (int c = 0; c < HD; c += 8) *reinterpret_cast<uint4*>(orow + c) = make_uint4(0, 0, 0, 0);
        if (p.lse != nullptr) p.lse[static_cast<size_t>(q_start + q0 + r) * p.HQ + h] = -INFINITY;
      }
    }
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_empty[i], kTcSoftmaxWarps);
      mbar_init(&bars->p_full[i], kTcSoftmaxWarps);
      mbar_init(&bars->pv_done[i], 1);
    }
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&tmq);
      prefetch_tensormap(&tmk);
      prefetch_tensormap(&tmv);
      mbar_arrive_expect_tx(&bars->q_full, Cfg::kTile);
#pragma unroll
      for (int db = 0; db < Cfg::kDBlk; ++db)
        tma_load_3d(sm + Cfg::kQ + db * Cfg::kBlk, &tmq, &bars->q_full, db * 64, h, q_start + q0);
      for (int t = 0; t < nkt && !*abort; ++t) {
        const int st = t % NS, use = t / NS;
        if (use > 0 && !tc_wait(&bars->k_empty[st], (use - 1) & 1, abort)) break;
        mbar_arrive_expect_tx(&bars->k_full[st], Cfg::kTile);
#pragma unroll
        for (int db = 0; db < Cfg::kDBlk; ++db)
          tma_load_3d(sm + Cfg::kK + st * Cfg::kTile + db * Cfg::kBlk, &tmk, &bars->k_full[st], db * 64, hk,
                      k_start + t * kTcKeys);
        if (use > 0 && !tc_wait(&bars->v_empty[st], (use - 1) & 1, abort)) break;
        mbar_arrive_expect_tx(&bars->v_full[st], Cfg::kTile);
#pragma unroll
        for (int db = 0; db < Cfg::kDBlk; ++db)
          tma_load_3d(sm + Cfg::kV + st * Cfg::kTile + db * Cfg::kBlk, &tmv, &bars->v_full[st], db * 64, hk,
                      k_start + t * kTcKeys);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc<T>(kTcRows, kTcKeys, false);
      constexpr uint32_t idesc_o = umma_idesc<T>(kTcRows, HD, true);
      const uint32_t q_base = smem_u32(sm + Cfg::kQ);
      auto issue_s = [&](int t) -> bool {
        const int sb = t & 1, st = t % NS;
        if (t >= 2 && !tc_wait(&bars->s_empty[sb], ((t >> 1) - 1) & 1, abort)) return false;
        if (!tc_wait(&bars->k_full[st], (t / NS) & 1, abort)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_u32(sm + Cfg::kK + st * Cfg::kTile);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * Cfg::kBlk + (kk & 3) * 32;
          umma_f16(tmem + sb * kTcKeys, smem_desc(q_base + off, 16, 1024), smem_desc(k_base + off, 16, 1024),
                   idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[sb]);
        umma_commit(&bars->k_empty[st]);
        return true;
      };
      bool ok = tc_wait(&bars->q_full, 0, abort);
      if (ok) ok = issue_s(0);
      for (int j = 0; j < nkt && ok; ++j) {
        if (j + 1 < nkt && !issue_s(j + 1)) break;
        const int pb = j & 1, vs = j % NS;
        if (!tc_wait(&bars->p_full[pb], (j >> 1) & 1, abort)) break;
        if (!tc_wait(&bars->v_full[vs], (j / NS) & 1, abort)) break;
        tc_fence_after();
        const uint32_t v_base = smem_u32(sm + Cfg::kV + vs * Cfg::kTile);
#pragma unroll
        for (int kk = 0; kk < kTcKeys / 16; ++kk) {
          const uint64_t vd = smem_desc(v_base + kk * 16 * 128, Cfg::kBlk, 1024);
          // 16 keys = 8 packed columns of the P buffer in tensor memory
          umma_f16_ts(tmem + Cfg::kTmemO, tmem + Cfg::kTmemP + pb * 64 + kk * 8, vd, idesc_o,
                      (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars->pv_done[pb]);
        umma_commit(&bars->v_empty[vs]);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    const int r = (warp - 4) * 32 + lane;  // query row within the tile == tensor-memory lane
    const int qi = q0 + r;                 // query index within the sequence
    const uint32_t lane_base = tmem + ((static_cast<uint32_t>(warp - 4) * 32u) << 16);
    const int vis_end = p.causal ? min(k_len, qi + shift + 1) : k_len;  // keys [0, vis_end) visible
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nkt; ++j) {
      const int sb = j & 1;
      // wait results are made warp-uniform: tcgen05.ld/st are warp-collective
      if (!__all_sync(0xffffffffu, tc_wait(&bars->s_full[sb], (j >> 1) & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kTcKeys];
#pragma unroll
      for (int c = 0; c < kTcKeys; c += 32) {
        uint32_t raw[32];
        tmem_ld32(lane_base + sb * kTcKeys + c, raw);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c + i] = __uint_as_float(raw[i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->s_empty[sb]);

      // scores into the log2 domain; masked keys become -inf (after scaling, so
      // a zero scale still gives -inf there and 0 elsewhere)
      const int key0 = j * kTcKeys;
      float mx = -INFINITY;
      if (key0 + kTcKeys <= vis_end) {
#pragma unroll
        for (int c = 0; c < kTcKeys; ++c) {
          s[c] *= p.scale_log2;
          mx = fmaxf(mx, s[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kTcKeys; ++c) {
          s[c] = (key0 + c < vis_end) ? s[c] * p.scale_log2 : -INFINITY;
          mx = fmaxf(mx, s[c]);
        }
      }
      const bool grow = mx > m_run + kRescaleThreshold;
      float alpha = 1.f;
      if (grow) {
        alpha = fast_exp2(m_run - mx);  // 0 when m_run = -inf
        m_run = mx;
        l_run *= alpha;
      }
      float rs = 0.f;
      uint32_t packed[kTcKeys / 2];
      if (m_run == -INFINITY) {
#pragma unroll
        for (int c = 0; c < kTcKeys / 2; ++c) packed[c] = 0u;
      } else {
#pragma unroll
        for (int c = 0; c < kTcKeys; c += 2) {
          const float p0 = fast_exp2(s[c] - m_run);
          const float p1 = fast_exp2(s[c + 1] - m_run);
          rs += p0 + p1;
          packed[c >> 1] = Elem<T>::pack(p0, p1);
        }
      }
      l_run += rs;

      // P buffer j%2 is free once P.V of tile j-2 finished; a rescale of O
      // additionally needs P.V of tile j-1 finished (O must be at rest).
      const bool warp_grow = __any_sync(0xffffffffu, grow) && j > 0;
      if (warp_grow) {
        if (!__all_sync(0xffffffffu, tc_wait(&bars->pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
          uint32_t o[32];
          tmem_ld32(lane_base + Cfg::kTmemO + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(lane_base + Cfg::kTmemO + c, o);
        }
      } else if (j >= 2) {
        if (!__all_sync(0xffffffffu, tc_wait(&bars->pv_done[sb], ((j - 2) >> 1) & 1, abort))) {
          ok = false;
          break;
        }
      }
      const uint32_t pt = lane_base + Cfg::kTmemP + sb * 64;
      tmem_st32(pt, *reinterpret_cast<const uint32_t(*)[32]>(&packed[0]));
      tmem_st32(pt + 32, *reinterpret_cast<const uint32_t(*)[32]>(&packed[32]));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[sb]);
    }

    // epilogue: O / l
    if (ok && __all_sync(0xffffffffu, tc_wait(&bars->pv_done[(nkt - 1) & 1], ((nkt - 1) >> 1) & 1, abort))) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      T* orow = outp + (static_cast<size_t>(q_start + qi) * p.HQ + h) * HD;
#pragma unroll
      for (int c = 0; c < HD; c += 32) {
        uint32_t o[32];
        tmem_ld32(lane_base + Cfg::kTmemO + c, o);
        if (qi < q_len) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 v;
            v.x = Elem<T>::pack(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv);
            v.y = Elem<T>::pack(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
            v.z = Elem<T>::pack(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
            v.w = Elem<T>::pack(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c + i) = v;
          }
        }
      }
      if (qi < q_len && p.lse != nullptr)
        p.lse[static_cast<size_t>(q_start + qi) * p.HQ + h] =
            l_run > 0.f ? (m_run + log2f(l_run)) * kLn2 : -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

}  // namespace mxfa
