// prefill_sm100.cuh -- attention forward on the 5th-generation tensor cores
// (tcgen05 MMA, accumulators in tensor memory, operands staged by TMA).
//
// CTA = one 128-row query tile of one head; 12 warps, specialised:
//   warp 0    : TMA producer -- Q once, then K and V tiles (128 keys) into
//               three-stage rings, in the order the tensor pipe consumes them
//   warp 1    : allocates tensor memory; issues the P.V products
//               O += P_j V_j (M=128, N=D, K=128; P from tensor memory, V MN-major)
//   warp 2    : issues the score products S_j = Q K_j^T (M=128, N=128, K=D)
//   warps 4-7 : softmax group 0 -- key tiles 0, 2, 4, ...
//   warps 8-11: softmax group 1 -- key tiles 1, 3, 5, ...
// Tensor memory: S/P buffers 0 | 1 | 2 (128 columns each) | O (D columns).
// Tile j uses buffer j % 3, so the score products of the next two tiles are
// ready while a group turns S_j into P_j (written over the columns of S_j it
// has read), and the two groups run consecutive tiles side by side.  Both
// accumulate into the one O with a running maximum they share through shared
// memory; the details are at prefill_tc_kernel below.
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

#define MXFA_RW32(x)                                                                                            \
  "+r"(x[0]), "+r"(x[1]), "+r"(x[2]), "+r"(x[3]), "+r"(x[4]), "+r"(x[5]), "+r"(x[6]), "+r"(x[7]), "+r"(x[8]),   \
      "+r"(x[9]), "+r"(x[10]), "+r"(x[11]), "+r"(x[12]), "+r"(x[13]), "+r"(x[14]), "+r"(x[15]), "+r"(x[16]),    \
      "+r"(x[17]), "+r"(x[18]), "+r"(x[19]), "+r"(x[20]), "+r"(x[21]), "+r"(x[22]), "+r"(x[23]), "+r"(x[24]),   \
      "+r"(x[25]), "+r"(x[26]), "+r"(x[27]), "+r"(x[28]), "+r"(x[29]), "+r"(x[30]), "+r"(x[31])

// Split load: the registers are written asynchronously and are valid only
// after tmem_wait_ld on the same array, whose read-write operands keep every
// use of them behind the wait.
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : MXFA_R32(r)
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : MXFA_RW32(r) : : "memory");
}
// Store without waiting; tmem_wait_st before the values are handed over.
__device__ __forceinline__ void tmem_st16_async(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      MXFA_W16(r)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 16 / 8 consecutive 32-bit columns (the masked softmax path works in
// 16-column chunks so its code stays small).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}

// Two fp32 lanes in one 64-bit register, for the packed fp32 instructions
// (fma/add .f32x2): one instruction per pair of scores in the softmax.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// P = 2^(s*scale - m) for 32 columns of one row: packed into 16 words of
// the element type, summed into two pair accumulators.
template <typename T>
__device__ __forceinline__ void exp2_chunk32(const uint32_t (&x)[32], uint64_t sc2, uint64_t nm2, uint64_t& acc0,
                                             uint64_t& acc1, uint32_t (&pk)[16]) {
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const uint64_t x01 = f2_fma(f2_pack(__uint_as_float(x[i]), __uint_as_float(x[i + 1])), sc2, nm2);
    const uint64_t x23 = f2_fma(f2_pack(__uint_as_float(x[i + 2]), __uint_as_float(x[i + 3])), sc2, nm2);
    float a, b, c, d;
    f2_unpack(x01, a, b);
    f2_unpack(x23, c, d);
    a = fast_exp2(a);
    b = fast_exp2(b);
    c = fast_exp2(c);
    d = fast_exp2(d);
    acc0 = f2_add(acc0, f2_pack(a, b));
    acc1 = f2_add(acc1, f2_pack(c, d));
    pk[i >> 1] = Elem<T>::pack(a, b);
    pk[(i >> 1) + 1] = Elem<T>::pack(c, d);
  }
}
// Row extreme (max for a positive scale, min for a negative one) of 32 columns, four chains.
__device__ __forceinline__ void ext_chunk32(const uint32_t (&x)[32], bool pos, float (&e)[4]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float v = __uint_as_float(x[i]);
    e[i & 3] = pos ? fmaxf(e[i & 3], v) : fminf(e[i & 3], v);
  }
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
constexpr int kTcGroupWarps = 4;  // warps per softmax group (one per tensor-memory lane quadrant)
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O when a row max grows by > 2^8

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

template <int HD>
struct TcCfg {
  // softmax groups of 4 warps (one per tensor-memory lane quadrant); group g
  // takes key tiles j with j % kGroups == g
  static constexpr int kGroups = 2;  // three groups measured no faster
  static constexpr int kThreads = (4 + 4 * kGroups) * 32;
  static constexpr int kDBlk = HD / 64;
  static constexpr int kStages = 3;
  static constexpr int kBlk = 128 * 128;               // one 64-column block of a 128-row tile
  static constexpr int kTile = kDBlk * kBlk;           // Q, K or V tile bytes
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kTile;
  static constexpr int kV = kK + kStages * kTile;
  static constexpr int kMl = kQ;                       // epilogue (m, l) exchange over Q once every product is done
  static constexpr int kMPub = kV + kStages * kTile;   // [2 parities][128 rows] running max handed between groups
  static constexpr int kBar = kMPub + 2 * kTcRows * 4;
  static constexpr int kNumBars = 1 + 2 * kStages + 3 * 3 + 2 * 4 + 1;
  static constexpr int kSmemBytes = kBar + kNumBars * 8 + 16 + 1024;
  static constexpr uint32_t kTmemCols = 512;           // S/P 0 | S/P 1 | S/P 2 | O
  static constexpr uint32_t kTmemO = 3 * kTcKeys;
  static constexpr int kSBufs = 3;
};

// K stage t%3 is released by S_t's completion (s_full) and V stage t%3 by
// P.V_t's (pv_done): one commit per product, each barrier read by every
// party that needs that product done.
template <int kStages>
struct TcBars {
  uint64_t q_full, k_full[kStages], v_full[kStages];
  uint64_t s_full[3], p_full[3], pv_done[3];
  uint64_t m_ready[2][4];  // [tile parity][warp quadrant]
  // Completes once, after the last P.V (and so every product): the epilogue
  // must not wait on a per-buffer barrier by parity, since a group that ran
  // out of tiles early can reach it two phases ahead of that barrier.
  uint64_t all_done;
};

// One output accumulator, three score buffers.  A layout with an O per
// softmax group (S0 | S1 | O0 | O1) fills tensor memory and forces the next
// score product into a buffer after the P.V product that reads the P stored
// there, so every group tile waits for its own softmax, one P.V and one score
// product in series.  With one O there is room for three S/P buffers: while a
// group turns S_j into P_j, S_{j+1} and S_{j+2} are already computed.
//
// One O means one running maximum per row for both groups.  The group of
// tile j reads m_{j-1} (published by the other group through shared memory,
// one mbarrier per warp quadrant and tile parity), raises it only when the
// tile's row maximum exceeds it by more than 2^8 (lazy rescale), and
// publishes m_j before its exp2 pass.  When m_j grew it rescales O in tensor
// memory after P.V_{j-1} completed and before P.V_j is issued (P.V_j waits
// for P_j, which this group has not released yet).  Each group keeps its own
// row sum at the maximum of its last tile; the epilogue brings both to the
// final maximum, which is also O's.
//
// The score and P.V products come from two issuing threads (warps 2 and 1):
// an issuing thread is held until the tensor pipe accepts each MMA, so one
// thread's waits and commits between chains left the pipe idle, while with
// two the other thread's chain fills those gaps.  Each product is committed
// once: s_full[b] (read by the softmax and by the producer, which then
// reloads that K stage) and pv_done[b] (read by the score issuer before it
// reuses buffer b, by the producer before it reloads that V stage, and by a
// rescaling softmax group).  No barrier is waited on more than one phase
// ahead of its state; the epilogue, which a group can reach while the last
// tile's buffer is still two phases behind, waits on a one-shot barrier.
//
// On a tile every row sees in full, the softmax reads S in 32-column loads
// whose wait is split from the load, so each load is in flight while the
// previous chunk is worked on; the last chunk of the maximum pass stays in
// registers and the exp2 pass's first load is issued before the maximum
// exchange.  The exp2 pass scales and sums two scores per instruction
// (fma/add .f32x2).  At the power cap fewer instructions are also a higher
// clock.
// kExactP: P is split into its rounded value and the rounded remainder,
// P_hi + P_lo (~16 significant bits), stored side by side in S's columns
// (per 16-key chunk: 8 columns of P_hi, then 8 of P_lo) and both multiplied
// with V, so P.V loses no precision to rounding P.  1.5x the tensor work;
// for inputs whose V has a wide dynamic range.
template <typename T, int HD, bool kExactP = false>
__global__ void __launch_bounds__(TcCfg<HD>::kThreads, 1)
    prefill_tc_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tmq,
                       const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv) {
  using Cfg = TcCfg<HD>;
  constexpr int NS = Cfg::kStages;
  constexpr int NB = Cfg::kSBufs;
  constexpr int NG = Cfg::kGroups;
  static_assert(2 * NG * kTcRows * 4 <= Cfg::kTile, "epilogue exchange fits the Q tile");
  static_assert(Cfg::kTmemO + HD <= Cfg::kTmemCols, "tensor memory layout");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  TcBars<NS>* bars = reinterpret_cast<TcBars<NS>*>(sm + Cfg::kBar);
  float* ml = reinterpret_cast<float*>(sm + Cfg::kMl);      // [group][m | l][row]
  float* mpub = reinterpret_cast<float*>(sm + Cfg::kMPub);  // [tile parity][row]
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
      mbar_init(&bars->v_full[i], 1);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], kTcGroupWarps);
      mbar_init(&bars->pv_done[i], 1);
    }
    for (int i = 0; i < 2; ++i)
      for (int qd = 0; qd < 4; ++qd) mbar_init(&bars->m_ready[i][qd], 32);
    mbar_init(&bars->all_done, 1);
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
      // Issue order = consumption order: K_0..K_2, then per tile V_t and K_{t+3}.
      // K_{t+3} replaces K_t once S_t is done; V_t replaces V_{t-3} once P.V_{t-3}
      // is done.  Neither copy ever waits behind a wait of the other kind that
      // the tensor pipe reaches later.
      auto load_k = [&](int t) {
        mbar_arrive_expect_tx(&bars->k_full[t % NS], Cfg::kTile);
#pragma unroll
        for (int db = 0; db < Cfg::kDBlk; ++db)
          tma_load_3d(sm + Cfg::kK + (t % NS) * Cfg::kTile + db * Cfg::kBlk, &tmk, &bars->k_full[t % NS], db * 64,
                      hk, k_start + t * kTcKeys);
      };
      for (int t = 0; t < NS && t < nkt; ++t) load_k(t);
      for (int t = 0; t < nkt && !*abort; ++t) {
        const int st = t % NS, use = t / NS;
        if (use > 0 && !tc_wait(&bars->pv_done[st], (use - 1) & 1, abort)) break;  // P.V_{t-3} done
        mbar_arrive_expect_tx(&bars->v_full[st], Cfg::kTile);
#pragma unroll
        for (int db = 0; db < Cfg::kDBlk; ++db)
          tma_load_3d(sm + Cfg::kV + st * Cfg::kTile + db * Cfg::kBlk, &tmv, &bars->v_full[st], db * 64, hk,
                      k_start + t * kTcKeys);
        if (t + NS < nkt) {
          if (!tc_wait(&bars->s_full[st], use & 1, abort)) break;  // S_t done with this stage
          load_k(t + NS);
        }
      }
    }
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------ MMA issue
    // Two issuing threads: warp 1 issues the P.V products, warp 2 the score
    // products.  An issuing thread is held until the tensor pipe accepts
    // each MMA, so with one thread every wait, commit and descriptor step
    // between two chains left the pipe idle; with two, one thread's chain
    // keeps the pipe busy while the other waits.  S_{t+3} reuses buffer t%3
    // only after P.V_t completed (pv_done), and P.V_t reads S_t's buffer only
    // after the softmax released P_t, which it does after S_t completed.
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc<T>(kTcRows, kTcKeys, false);
      constexpr uint32_t idesc_o = umma_idesc<T>(kTcRows, HD, true);
      constexpr int kS = HD / 16;        // K-steps of a score product
      constexpr int kP = kTcKeys / 16;   // K-steps of a P.V product
      if (warp == 2) {
        auto s_step = [](int kk) -> uint64_t { return (kk >> 2) * (Cfg::kBlk >> 4) + (kk & 3) * 2; };
        uint64_t qd[kS];
        {
          const uint64_t base = smem_desc(smem_u32(sm + Cfg::kQ), 16, 1024);
#pragma unroll
          for (int kk = 0; kk < kS; ++kk) qd[kk] = base + s_step(kk);
        }
        bool ok = tc_wait(&bars->q_full, 0, abort);
        for (int t = 0; t < nkt && ok; ++t) {
          const int buf = t % NB, ks = t % NS;
          uint64_t kd[kS];
          {
            const uint64_t base = smem_desc(smem_u32(sm + Cfg::kK + ks * Cfg::kTile), 16, 1024);
#pragma unroll
            for (int kk = 0; kk < kS; ++kk) kd[kk] = base + s_step(kk);
          }
          pin_regs(kd);
          if (t >= NB && !tc_wait(&bars->pv_done[buf], ((t - NB) / NB) & 1, abort)) break;  // buffer free
          if (!tc_wait(&bars->k_full[ks], (t / NS) & 1, abort)) break;
          tc_fence_after();
          umma_ss_chain(tmem + buf * kTcKeys, qd, kd, idesc_s);
          umma_commit(&bars->s_full[buf]);
        }
      } else {
        for (int j = 0; j < nkt; ++j) {
          const int buf = j % NB, vs = j % NS;
          uint64_t vd[kP];
          uint32_t pa[kP], pl[kP];
          {
            const uint64_t vbase = smem_desc(smem_u32(sm + Cfg::kV + vs * Cfg::kTile), Cfg::kBlk, 1024);
#pragma unroll
            for (int kk = 0; kk < kP; ++kk) {
              vd[kk] = vbase + kk * (16 * 128 >> 4);
              // P_j packed over the columns of S_j: 8 columns per 16 keys, or
              // (exact P) P_hi then P_lo in the 16 columns of each 16 keys
              pa[kk] = tmem + buf * kTcKeys + (kExactP ? kk * 16 : kk * 8);
              pl[kk] = pa[kk] + 8;
            }
          }
          pin_regs(vd);
          pin_regs(pa);
          if (!tc_wait(&bars->v_full[vs], (j / NS) & 1, abort)) break;
          if (!tc_wait(&bars->p_full[buf], (j / NB) & 1, abort)) break;
          tc_fence_after();
          umma_ts_chain(tmem + Cfg::kTmemO, pa, vd, idesc_o, j > 0 ? 1u : 0u);
          if constexpr (kExactP) umma_ts_chain(tmem + Cfg::kTmemO, pl, vd, idesc_o, 1u);
          umma_commit(&bars->pv_done[buf]);
          // every score product completed before P_{nkt-1} existed, so this
          // marks the end of all tensor-memory and shared-memory reads
          if (j == nkt - 1) umma_commit(&bars->all_done);
        }
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    const int g = (warp - 4) >> 2;          // group: key tiles j with j % NG == g
    const int quad = warp & 3;              // tensor-memory lane quadrant
    const int r = quad * 32 + lane;         // query row within the tile == tensor-memory lane
    const int qi = q0 + r;                  // query index within the sequence
    const uint32_t lane_base = tmem + ((static_cast<uint32_t>(quad) * 32u) << 16);
    const uint32_t o_base = lane_base + Cfg::kTmemO;
    const int vis_end = p.causal ? min(k_len, qi + shift + 1) : k_len;  // keys [0, vis_end) visible
    const float sc = p.scale_log2;
    float m_own = -INFINITY, l_own = 0.f;   // this group's row sum, at the maximum of its last tile
    bool ok = true;
    for (int j = g; j < nkt; j += NG) {
      const int buf = j % NB;
      if (!__all_sync(0xffffffffu, tc_wait(&bars->s_full[buf], (j / NB) & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sbuf = lane_base + buf * kTcKeys;
      const int key0 = j * kTcKeys;
      const bool full = key0 + kTcKeys <= vis_end;

      // pass 1: the row's extreme raw score over visible keys (max for a
      // positive scale, min for a negative one), scaled into the log2 domain
      const bool all_full = __all_sync(0xffffffffu, full);
      const bool pos = sc >= 0.f;
      const float ext0 = pos ? -INFINITY : INFINITY;
      float ext = ext0;
      uint32_t ra[32], rb[32];
      if (all_full) {
        // 32-column loads, each in flight while the previous chunk is
        // compared (four chains).  The last chunk stays in registers for
        // pass 2, whose first load goes out before the maximum exchange.
        float e[4] = {ext0, ext0, ext0, ext0};
        tmem_ld32_async(sbuf, ra);
        tmem_wait_ld(ra);
        tmem_ld32_async(sbuf + 32, rb);
        ext_chunk32(ra, pos, e);
        tmem_wait_ld(rb);
        tmem_ld32_async(sbuf + 64, ra);
        ext_chunk32(rb, pos, e);
        tmem_wait_ld(ra);
        tmem_ld32_async(sbuf + 96, rb);
        ext_chunk32(ra, pos, e);
        tmem_wait_ld(rb);
        if constexpr (!kExactP) tmem_ld32_async(sbuf, ra);
        ext_chunk32(rb, pos, e);
        ext = pos ? fmaxf(fmaxf(e[0], e[1]), fmaxf(e[2], e[3])) : fminf(fminf(e[0], e[1]), fminf(e[2], e[3]));
      } else {
        // diagonal tile: a rolled loop over 16-column chunks keeps this
        // rarely taken path out of the way of the unrolled one
#pragma unroll 1
        for (int c = 0; c < kTcKeys; c += 16) {
          uint32_t raw[16];
          tmem_ld16(sbuf + c, raw);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float v = __uint_as_float(raw[i]);
            const bool vis = key0 + c + i < vis_end;
            ext = vis ? (pos ? fmaxf(ext, v) : fminf(ext, v)) : ext;
          }
        }
      }
      const float mx = (ext == INFINITY || ext == -INFINITY) ? -INFINITY : ext * sc;

      // the running maximum after tile j-1, from the other group
      float m_in = -INFINITY;
      if (j > 0) {
        const int pj = j - 1;
        if (!__all_sync(0xffffffffu, tc_wait(&bars->m_ready[pj & 1][quad], (pj >> 1) & 1, abort))) {
          ok = false;
          break;
        }
        m_in = mpub[(pj & 1) * kTcRows + r];
      }
      const float m_j = mx > m_in + kRescaleThreshold ? mx : m_in;
      // every lane releases its own row's value (arrival count 32)
      mpub[(j & 1) * kTcRows + r] = m_j;
      mbar_arrive(&bars->m_ready[j & 1][quad]);

      if (m_j != m_own) {  // this group's sum follows the maximum it now uses
        l_own *= fast_exp2(m_own - m_j);  // 0 when m_own = -inf
        m_own = m_j;
      }
      // O holds tiles < j at m_in; bring it to m_j once P.V_{j-1} is done
      // (P.V_j cannot start before this group releases P_j)
      const bool grow = j > 0 && m_j != m_in;
      if (__any_sync(0xffffffffu, grow)) {
        const int pj = j - 1;
        if (!__all_sync(0xffffffffu, tc_wait(&bars->pv_done[pj % NB], (pj / NB) & 1, abort))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float alpha = grow ? fast_exp2(m_in - m_j) : 1.f;  // 0 when m_in = -inf
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
          uint32_t o[32];
          tmem_ld32(o_base + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(o_base + c, o);
        }
      }

      // pass 2: P = 2^(s*scale - m_j), packed in pairs into columns of S
      // that were already read
      float rs = 0.f;
      const float neg_m = -m_j;
      if (kExactP && all_full) {
        // 64-key halves read at once; per 16-key chunk, P_hi then P_lo in the
        // chunk's own (already read) columns, stored 32 columns at a time
        float r0 = 0.f, r1 = 0.f;
#pragma unroll 1
        for (int c = 0; c < kTcKeys; c += 64) {
          uint32_t raw[64];
          tmem_ld64(sbuf + c, raw);
#pragma unroll
          for (int qq = 0; qq < 2; ++qq) {
            uint32_t packed[32];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const float p0 = fast_exp2(fmaf(__uint_as_float(raw[32 * qq + i]), sc, neg_m));
              const float p1 = fast_exp2(fmaf(__uint_as_float(raw[32 * qq + i + 1]), sc, neg_m));
              r0 += p0;
              r1 += p1;
              const uint32_t hi = Elem<T>::pack(p0, p1);
              const float2 hf = Elem<T>::unpack(hi);
              const int w = (i >> 4) * 16 + ((i & 15) >> 1);  // chunk i/16: hi words 0-7, lo words 8-15
              packed[w] = hi;
              packed[w + 8] = Elem<T>::pack(p0 - hf.x, p1 - hf.y);
            }
            tmem_st32(sbuf + c + 32 * qq, packed);
          }
        }
        rs = r0 + r1;
      } else if constexpr (kExactP) {
        // diagonal tile, 16-key chunks: P_hi and P_lo land in the chunk's own (already read) columns
        const bool live = m_j != -INFINITY;
#pragma unroll 1
        for (int c = 0; c < kTcKeys; c += 16) {
          uint32_t raw[16];
          tmem_ld16(sbuf + c, raw);
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const bool v0 = live && (all_full || key0 + c + i < vis_end);
            const bool v1 = live && (all_full || key0 + c + i + 1 < vis_end);
            const float p0 = v0 ? fast_exp2(fmaf(__uint_as_float(raw[i]), sc, neg_m)) : 0.f;
            const float p1 = v1 ? fast_exp2(fmaf(__uint_as_float(raw[i + 1]), sc, neg_m)) : 0.f;
            rs += p0 + p1;
            const uint32_t hi = Elem<T>::pack(p0, p1);
            const float2 hf = Elem<T>::unpack(hi);
            packed[i >> 1] = hi;
            packed[8 + (i >> 1)] = Elem<T>::pack(p0 - hf.x, p1 - hf.y);
          }
          tmem_st16(sbuf + c, packed);
        }
      } else if (all_full) {  // every row sees every key of the tile, so m_j is finite
        // rb holds columns 96-127 from pass 1 and ra's load of columns 0-31
        // is in flight; each later load overlaps the previous chunk's exp2.
        // P of columns [32k, 32k+32) goes to columns [16k, 16k+16), which
        // lie in columns already read; the stores are waited on once.
        const uint64_t sc2 = f2_pack(sc, sc), nm2 = f2_pack(neg_m, neg_m);
        uint64_t acc0 = 0, acc1 = 0;  // four sum chains: columns i % 4
        uint32_t pk3[16], pka[16], pkb[16];
        exp2_chunk32<T>(rb, sc2, nm2, acc0, acc1, pk3);
        tmem_wait_ld(ra);
        tmem_ld32_async(sbuf + 32, rb);
        exp2_chunk32<T>(ra, sc2, nm2, acc0, acc1, pka);
        tmem_st16_async(sbuf, pka);
        tmem_wait_ld(rb);
        tmem_ld32_async(sbuf + 64, ra);
        exp2_chunk32<T>(rb, sc2, nm2, acc0, acc1, pkb);
        tmem_st16_async(sbuf + 16, pkb);
        tmem_st16_async(sbuf + 48, pk3);  // columns 48-63 were read with chunk 1
        tmem_wait_ld(ra);
        tmem_wait_st();  // pka is written again below
        exp2_chunk32<T>(ra, sc2, nm2, acc0, acc1, pka);
        tmem_st16_async(sbuf + 32, pka);
        tmem_wait_st();
        float a, bb;
        f2_unpack(f2_add(acc0, acc1), a, bb);
        rs = a + bb;
      } else {
        const bool live = m_j != -INFINITY;
#pragma unroll 1
        for (int c = 0; c < kTcKeys; c += 16) {
          uint32_t raw[16];
          tmem_ld16(sbuf + c, raw);
          uint32_t packed[8];
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const bool v0 = live && key0 + c + i < vis_end;
            const bool v1 = live && key0 + c + i + 1 < vis_end;
            const float p0 = v0 ? fast_exp2(fmaf(__uint_as_float(raw[i]), sc, neg_m)) : 0.f;
            const float p1 = v1 ? fast_exp2(fmaf(__uint_as_float(raw[i + 1]), sc, neg_m)) : 0.f;
            rs += p0 + p1;
            packed[i >> 1] = Elem<T>::pack(p0, p1);
          }
          // P columns [c/2, c/2 + 8) lie in the S columns already read
          tmem_st8(sbuf + (c >> 1), packed);
        }
      }
      l_own += rs;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[buf]);
    }
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");  // a load left in flight by an aborted tile

    // ---------------------------------------------------------- merge + store
    // Every product is complete once the last P.V is; the Q tile's shared
    // memory is then free for the (m, l) exchange.
    const bool done_ok = __all_sync(0xffffffffu, ok && tc_wait(&bars->all_done, 0, abort));
    fence_proxy_async_smem();
    ml[(g * 2) * kTcRows + r] = m_own;
    ml[(g * 2 + 1) * kTcRows + r] = l_own;
    named_barrier_sync(1, NG * kTcGroupWarps * 32);
    if (done_ok) {
      tc_fence_after();
      float M = -INFINITY;  // the last tile's maximum, at which O is held
#pragma unroll
      for (int gg = 0; gg < NG; ++gg) M = fmaxf(M, ml[(gg * 2) * kTcRows + r]);
      float L = 0.f;
#pragma unroll
      for (int gg = 0; gg < NG; ++gg) {
        const float mg = ml[(gg * 2) * kTcRows + r];
        if (mg != -INFINITY) L += ml[(gg * 2 + 1) * kTcRows + r] * fast_exp2(mg - M);
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      T* orow = outp + (static_cast<size_t>(q_start + qi) * p.HQ + h) * HD;
      // group g stores the 32-column chunks g, g + NG, ...
      for (int c = g * 32; c < HD; c += NG * 32) {
        uint32_t o[32];
        tmem_ld32(o_base + c, o);
        if (qi < q_len) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 v;
            v.x = Elem<T>::pack(__uint_as_float(o[i + 0]) * inv, __uint_as_float(o[i + 1]) * inv);
            v.y = Elem<T>::pack(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
            v.z = Elem<T>::pack(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
            v.w = Elem<T>::pack(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
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
