// prefill_sm100.cuh -- attention forward on the 5th-generation tensor cores
// (tcgen05 MMA, accumulators in tensor memory, operands staged by TMA).
//
// CTA = one 128-row query tile of one head; 12 warps, specialised:
//   warp 0    : TMA producer -- Q once, then K and V tiles (128 keys) into a
//               three-stage ring, each stage guarded by full/empty mbarriers
//   warp 1    : allocates tensor memory and issues every tcgen05.mma from one
//               thread:  S_j = Q K_j^T   (M=128, N=128, K=D; both K-major)
//                        O_{j%2} += P_j V_j (M=128, N=D, K=128; P from tensor
//                        memory, V MN-major), committing each to an mbarrier
//   warps 4-7 : softmax group 0 -- key tiles 0, 2, 4, ...
//   warps 8-11: softmax group 1 -- key tiles 1, 3, 5, ...
// Each softmax group keeps its own online state (m, l) and its own output
// accumulator O_g in tensor memory, like two interleaved splits of the key
// range; the groups merge (m, l, O) once at the end.  Two groups put two
// softmax warps on every SM sub-partition, so one warp's exp2 / conversion
// latency overlaps the other's work, and the tensor pipe always has the other
// group's products queued.  Per tile a group makes two passes over S in
// tensor memory (row max, then exp2 + sum + bf16/fp16 pack), writing P_j over
// the columns of S_j it has already read.
// Tensor memory: S/P buffer 0 | S/P buffer 1 | O_0 | O_1 (128 + 128 + 2*D columns).
// The next score product into a buffer is issued after the P.V product that
// reads it; tcgen05.mma from one thread execute in issue order.
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

// A chain of MMAs into one accumulator, issued from one asm block: descriptors
// (and tensor-memory A addresses) are computed by the caller ahead of time,
// so issuing is back-to-back tcgen05.mma instructions.  The first MMA of an
// SS chain starts the accumulator; a TS chain's first MMA accumulates when
// `acc` is non-zero; every later MMA accumulates.
__device__ __forceinline__ void umma_ss_chain(uint32_t d, const uint64_t (&a)[8], const uint64_t (&b)[8],
                                              uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred pf, pt;\n\t"
      "setp.ne.b32 pf, %17, %17;\n\tsetp.eq.b32 pt, %17, %17;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %9, %17, pf;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %10, %17, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %11, %17, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %12, %17, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %5, %13, %17, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %6, %14, %17, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %7, %15, %17, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %8, %16, %17, pt;\n\t}" ::"r"(d),
      "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(b[0]),
      "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "r"(idesc)
      : "memory");
}
__device__ __forceinline__ void umma_ss_chain(uint32_t d, const uint64_t (&a)[4], const uint64_t (&b)[4],
                                              uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred pf, pt;\n\t"
      "setp.ne.b32 pf, %9, %9;\n\tsetp.eq.b32 pt, %9, %9;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %5, %9, pf;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %6, %9, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %7, %9, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %8, %9, pt;\n\t}" ::"r"(d),
      "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "r"(idesc)
      : "memory");
}
__device__ __forceinline__ void umma_ts_chain(uint32_t d, const uint32_t (&a)[8], const uint64_t (&b)[8],
                                              uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred pa, pt;\n\t"
      "setp.ne.b32 pa, %18, 0;\n\tsetp.eq.b32 pt, %17, %17;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %9, %17, pa;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %10, %17, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %11, %17, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %12, %17, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], %13, %17, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%6], %14, %17, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], %15, %17, pt;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%8], %16, %17, pt;\n\t}" ::"r"(d),
      "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7]), "l"(b[0]),
      "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "r"(idesc), "r"(acc)
      : "memory");
}

// Make values opaque to the compiler at this point, so they are computed
// here (ahead of a wait) and not re-derived next to their use.
template <int N>
__device__ __forceinline__ void pin_regs(uint64_t (&x)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+l"(x[i]));
}
template <int N>
__device__ __forceinline__ void pin_regs(uint32_t (&x)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(x[i]));
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

#define MXFA_R64(x)                                                                                             \
  MXFA_R32(x), "=r"(x[32]), "=r"(x[33]), "=r"(x[34]), "=r"(x[35]), "=r"(x[36]), "=r"(x[37]), "=r"(x[38]),       \
      "=r"(x[39]), "=r"(x[40]), "=r"(x[41]), "=r"(x[42]), "=r"(x[43]), "=r"(x[44]), "=r"(x[45]), "=r"(x[46]),   \
      "=r"(x[47]), "=r"(x[48]), "=r"(x[49]), "=r"(x[50]), "=r"(x[51]), "=r"(x[52]), "=r"(x[53]), "=r"(x[54]),   \
      "=r"(x[55]), "=r"(x[56]), "=r"(x[57]), "=r"(x[58]), "=r"(x[59]), "=r"(x[60]), "=r"(x[61]), "=r"(x[62]),   \
      "=r"(x[63])

// 64 consecutive columns in one load (one wait).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,"
      "%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : MXFA_R64(r)
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

#define MXFA_W16(x)                                                                                             \
  "r"(x[0]), "r"(x[1]), "r"(x[2]), "r"(x[3]), "r"(x[4]), "r"(x[5]), "r"(x[6]), "r"(x[7]), "r"(x[8]), "r"(x[9]), \
      "r"(x[10]), "r"(x[11]), "r"(x[12]), "r"(x[13]), "r"(x[14]), "r"(x[15])

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      MXFA_W16(r)
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
constexpr int kTcThreads = 384;
constexpr int kTcGroupWarps = 4;  // warps per softmax group (one per tensor-memory lane quadrant)
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
  static constexpr int kMl = kQ;                       // merge scratch over Q once every product is done
  static constexpr int kBar = kV + kStages * kTile;
  static constexpr int kNumBars = 1 + 4 * kStages + 6;
  static constexpr int kSmemBytes = kBar + kNumBars * 8 + 16 + 1024;
  static constexpr uint32_t kTmemCols = 512;           // S/P 0 | S/P 1 | O_0 | O_1
  static constexpr uint32_t kTmemO = 2 * kTcKeys;      // O_g at kTmemO + g * HD
};

template <int kStages>
struct TcBars {
  uint64_t q_full, k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
  uint64_t s_full[2], p_full[2], pv_done[2];
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
  float* ml = reinterpret_cast<float*>(sm + Cfg::kMl);  // [group][m | l][row]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Cfg::kBar + Cfg::kNumBars * 8);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // Grid: x = query head, y = sequence, z = query tile (slowest).  Blocks go
  // out in linear order, so every head and sequence's latest (heaviest, for
  // causal) tiles start before any lighter tile: heaviest first across the
  // whole grid, which leaves only light tiles for the tail.
  const int h = blockIdx.x;
  const int b = blockIdx.y;
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
  const int qt = gridDim.z - 1 - blockIdx.z;
  const int q0 = qt * kTcRows;
  if (q0 >= q_len) return;
  const int shift = k_len - q_len;
  const int last_row = min(q0 + kTcRows, q_len) - 1;
  const int k_end = p.causal ? min(k_len, last_row + shift + 1) : k_len;
  const int nkt = k_end > 0 ? (k_end + kTcKeys - 1) / kTcKeys : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  T* outp = static_cast<T*>(p.out);
  if (nkt == 0) {  // every row of this tile sees no key: output 0, LSE -inf
    if (warp >= 4 && warp < 8) {
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
      mbar_init(&bars->p_full[i], kTcGroupWarps);
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
      constexpr int kS = HD / 16;        // K-steps of a score product
      constexpr int kP = kTcKeys / 16;   // K-steps of a P.V product
      // Descriptor start addresses are in 16-byte units (bits 0-13) and every
      // operand lies inside shared memory, so a step is a plain add.  Q and K
      // (K-major) advance 32 bytes per 16-column step within a 128-byte row
      // and a whole 64-column block every four steps; V (MN-major) advances 16
      // key rows = 2 KB per step.
      auto s_step = [](int kk) -> uint64_t { return (kk >> 2) * (Cfg::kBlk >> 4) + (kk & 3) * 2; };
      uint64_t qd[kS];
      {
        const uint64_t base = smem_desc(smem_u32(sm + Cfg::kQ), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < kS; ++kk) qd[kk] = base + s_step(kk);
      }
      auto k_descs = [&](int st, uint64_t (&kd)[kS]) {
        const uint64_t base = smem_desc(smem_u32(sm + Cfg::kK + st * Cfg::kTile), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < kS; ++kk) kd[kk] = base + s_step(kk);
      };
      bool ok = tc_wait(&bars->q_full, 0, abort);
      for (int t = 0; t < 2 && t < nkt && ok; ++t) {
        uint64_t kd[kS];
        k_descs(t % NS, kd);
        const int st = t % NS;
        if (!tc_wait(&bars->k_full[st], (t / NS) & 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        umma_ss_chain(tmem + t * kTcKeys, qd, kd, idesc_s);
        umma_commit(&bars->s_full[t]);
        umma_commit(&bars->k_empty[st]);
      }
      for (int j = 0; j < nkt && ok; ++j) {
        const int pb = j & 1, vs = j % NS, ks = (j + 2) % NS;
        const bool next_s = j + 2 < nkt;
        // everything the two products need is computed before the waits
        uint64_t vd[kP], kd[kS];
        uint32_t pa[kP];
        {
          const uint64_t vbase = smem_desc(smem_u32(sm + Cfg::kV + vs * Cfg::kTile), Cfg::kBlk, 1024);
#pragma unroll
          for (int kk = 0; kk < kP; ++kk) {
            vd[kk] = vbase + kk * (16 * 128 >> 4);
            // 16 keys = 8 packed columns of P_j (written over S_j in buffer j%2)
            pa[kk] = tmem + pb * kTcKeys + kk * 8;
          }
        }
        k_descs(ks, kd);
        pin_regs(vd);
        pin_regs(kd);
        pin_regs(pa);
        // K_{j+2} and V_j landed long before P_j is ready: wait for them
        // first, so nothing but P_j stands between the softmax and the two
        // products
        if (next_s && !tc_wait(&bars->k_full[ks], ((j + 2) / NS) & 1, abort)) break;
        if (!tc_wait(&bars->v_full[vs], (j / NS) & 1, abort)) break;
        if (!tc_wait(&bars->p_full[pb], (j >> 1) & 1, abort)) break;
        tc_fence_after();
        umma_ts_chain(tmem + Cfg::kTmemO + pb * HD, pa, vd, idesc_o, j >= 2 ? 1u : 0u);
        // S_{j+2} reuses buffer j%2; it is issued after the P.V product above
        if (next_s) umma_ss_chain(tmem + pb * kTcKeys, qd, kd, idesc_s);
        // each commit tracks every product issued before it
        if (next_s) {
          umma_commit(&bars->s_full[pb]);
          umma_commit(&bars->k_empty[ks]);
        }
        umma_commit(&bars->pv_done[pb]);
        umma_commit(&bars->v_empty[vs]);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    const int g = (warp - 4) >> 2;          // group: key tiles j with j % 2 == g
    const int quad = warp & 3;              // tensor-memory lane quadrant
    const int r = quad * 32 + lane;         // query row within the tile == tensor-memory lane
    const int qi = q0 + r;                  // query index within the sequence
    const uint32_t lane_base = tmem + ((static_cast<uint32_t>(quad) * 32u) << 16);
    const uint32_t o_base = lane_base + Cfg::kTmemO + g * HD;
    const int vis_end = p.causal ? min(k_len, qi + shift + 1) : k_len;  // keys [0, vis_end) visible
    const float sc = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = g; j < nkt; j += 2) {
      // wait results are made warp-uniform: tcgen05.ld/st are warp-collective
      if (!__all_sync(0xffffffffu, tc_wait(&bars->s_full[g], (j >> 1) & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sbuf = lane_base + g * kTcKeys;
      const int key0 = j * kTcKeys;
      const bool full = key0 + kTcKeys <= vis_end;

      // pass 1: the row's extreme raw score over visible keys (max for a
      // positive scale, min for a negative one), scaled into the log2 domain
      const bool all_full = __all_sync(0xffffffffu, full);
      const bool pos = sc >= 0.f;
      float ext = pos ? -INFINITY : INFINITY;
#pragma unroll
      for (int c = 0; c < kTcKeys; c += 64) {
        uint32_t raw[64];
        tmem_ld64(sbuf + c, raw);
        if (all_full) {
          float e0 = ext, e1 = pos ? -INFINITY : INFINITY;
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            e0 = pos ? fmaxf(e0, __uint_as_float(raw[i])) : fminf(e0, __uint_as_float(raw[i]));
            e1 = pos ? fmaxf(e1, __uint_as_float(raw[i + 1])) : fminf(e1, __uint_as_float(raw[i + 1]));
          }
          ext = pos ? fmaxf(e0, e1) : fminf(e0, e1);
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const float v = __uint_as_float(raw[i]);
            const bool vis = key0 + c + i < vis_end;
            ext = vis ? (pos ? fmaxf(ext, v) : fminf(ext, v)) : ext;
          }
        }
      }
      const float mx = (ext == INFINITY || ext == -INFINITY) ? -INFINITY : ext * sc;
      const bool grow = mx > m_run + kRescaleThreshold;
      float alpha = 1.f;
      if (grow) {
        alpha = fast_exp2(m_run - mx);  // 0 when m_run = -inf
        m_run = mx;
        l_run *= alpha;
      }
      // O_g last received P.V of tile j-2, which completed before S_j (same
      // issuing thread), so it is at rest here; rescale it when a row max grew
      if (__any_sync(0xffffffffu, grow) && j >= 2) {
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
          uint32_t o[32];
          tmem_ld32(o_base + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(o_base + c, o);
        }
      }

      // pass 2: P = 2^(s*scale - m) over each 64-key half, packed in pairs into
      // the 32 columns of S that the halves before it already consumed
      float rs = 0.f;
      const float neg_m = -m_run;
      const bool live = m_run != -INFINITY;
#pragma unroll
      for (int c = 0; c < kTcKeys; c += 64) {
        uint32_t raw[64];
        tmem_ld64(sbuf + c, raw);
        uint32_t packed[32];
        if (all_full && live) {
          float r0 = 0.f, r1 = 0.f;
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            const float p0 = fast_exp2(fmaf(__uint_as_float(raw[i]), sc, neg_m));
            const float p1 = fast_exp2(fmaf(__uint_as_float(raw[i + 1]), sc, neg_m));
            r0 += p0;
            r1 += p1;
            packed[i >> 1] = Elem<T>::pack(p0, p1);
          }
          rs += r0 + r1;
        } else {
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            const bool v0 = live && key0 + c + i < vis_end;
            const bool v1 = live && key0 + c + i + 1 < vis_end;
            const float p0 = v0 ? fast_exp2(fmaf(__uint_as_float(raw[i]), sc, neg_m)) : 0.f;
            const float p1 = v1 ? fast_exp2(fmaf(__uint_as_float(raw[i + 1]), sc, neg_m)) : 0.f;
            rs += p0 + p1;
            packed[i >> 1] = Elem<T>::pack(p0, p1);
          }
        }
        tmem_st32(sbuf + (c >> 1), packed);
      }
      l_run += rs;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[g]);
    }

    // ---------------------------------------------------------- merge + store
    // Both accumulators must be complete; the last P.V is the last product,
    // so afterwards the Q tile's shared memory is free for the (m, l) exchange.
    bool done_ok = ok;
#pragma unroll
    for (int gg = 0; gg < 2; ++gg) {
      if (nkt > gg) {
        const int jl = gg + ((nkt - 1 - gg) >> 1) * 2;  // last tile of parity gg
        done_ok = __all_sync(0xffffffffu, done_ok && tc_wait(&bars->pv_done[gg], (jl >> 1) & 1, abort));
      }
    }
    fence_proxy_async_smem();
    ml[(g * 2) * kTcRows + r] = m_run;
    ml[(g * 2 + 1) * kTcRows + r] = l_run;
    named_barrier_sync(1, 2 * kTcGroupWarps * 32);
    if (done_ok) {
      tc_fence_after();
      const float m0 = ml[r], l0 = ml[kTcRows + r];
      const float m1 = ml[2 * kTcRows + r], l1 = ml[3 * kTcRows + r];
      const float M = fmaxf(m0, m1);
      const float a0 = m0 != -INFINITY ? fast_exp2(m0 - M) : 0.f;
      const float a1 = m1 != -INFINITY ? fast_exp2(m1 - M) : 0.f;
      const float L = l0 * a0 + l1 * a1;
      const float inv = L > 0.f ? 1.f / L : 0.f;
      const float w0 = a0 * inv, w1 = a1 * inv;
      const bool two = nkt > 1;
      T* orow = outp + (static_cast<size_t>(q_start + qi) * p.HQ + h) * HD;
      // group g stores columns [g*HD/2, (g+1)*HD/2)
#pragma unroll
      for (int c = g * (HD / 2); c < (g + 1) * (HD / 2); c += 32) {
        uint32_t o0[32], o1[32];
        tmem_ld32(lane_base + Cfg::kTmemO + c, o0);
        if (two) tmem_ld32(lane_base + Cfg::kTmemO + HD + c, o1);
        if (qi < q_len) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float x0 = w0 > 0.f ? __uint_as_float(o0[i + e]) * w0 : 0.f;
              const float x1 = (two && w1 > 0.f) ? __uint_as_float(o1[i + e]) * w1 : 0.f;
              f[e] = x0 + x1;
            }
            uint4 v;
            v.x = Elem<T>::pack(f[0], f[1]);
            v.y = Elem<T>::pack(f[2], f[3]);
            v.z = Elem<T>::pack(f[4], f[5]);
            v.w = Elem<T>::pack(f[6], f[7]);
            *reinterpret_cast<uint4*>(orow + c + i) = v;
          }
        }
      }
      if (g == 0 && qi < q_len && p.lse != nullptr)
        p.lse[static_cast<size_t>(q_start + qi) * p.HQ + h] = L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
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
