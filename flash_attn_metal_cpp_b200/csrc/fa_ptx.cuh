// fa_ptx.cuh - thin inline-PTX wrappers for the sm_100a primitives used by
// the attention kernels: mbarriers, TMA tile loads, tcgen05 (TMEM alloc,
// MMA, commit, ld/st, fences) and shared-memory matrix descriptors.
//
// Every wait in this file is bounded: fa_wait() gives up after a wall-clock
// limit read from %globaltimer, records FA_DEV_TIMEOUT in the device status
// word and returns false, so a kernel never spins forever.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace fa {

// Status bits written by kernels into the per-device status word.
enum : unsigned {
  FA_DEV_TIMEOUT = 1u,
};

// Default wall-clock limit of any single in-kernel wait (nanoseconds). A
// correct wait lasts microseconds; this only ends a kernel whose partner is
// gone. Callers can set another limit (fa_set_wait_limit); kernels take it
// from AttnArgs::wait_limit_ns.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint (ns): the thread sleeps in hardware until
// the phase completes or the hint elapses, instead of spinning and taking
// issue slots from the warps that do the work.
constexpr uint32_t kSuspendHintNs = 1000000u;
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Wait until the phase with parity `parity` of barrier `bar` has completed.
// Returns false (and records a timeout in *status) if `limit_ns` ran out.
__device__ __forceinline__ bool fa_wait(uint32_t bar, uint32_t parity, unsigned* status,
                                        unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) {
      atomicOr(status, FA_DEV_TIMEOUT);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
// 4-D tiled bulk tensor load global -> shared, completion counted in bytes
// on `bar`. Each CTA loads its own tiles (no cluster sharing).
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, uint32_t bar, int c0,
                                            int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ------------------------------------------------ programmatic dependent launch
// Kernels launched with launch_pdl may start while the kernel before them in
// the stream is still running. grid_dep_wait() blocks the calling thread until
// that kernel has completed and its memory is visible; every thread calls it
// before its first global-memory access. grid_dep_launch_dependents() lets
// the next such kernel start launching (it still waits in grid_dep_wait).
// Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T-ish per the instruction descriptor.
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same as mma_ss with each descriptor given as (low word, high word): the
// caller keeps the high words constant and advances only the start-address
// field in the low words, so issuing an MMA costs two integer adds.
__device__ __forceinline__ void mma_ss_lohi(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo,
                                            uint32_t b_hi, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 ad, bd;\n\t"
      "mov.b64 ad, {%1, %2};\n\t"
      "mov.b64 bd, {%3, %4};\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %5, p;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_ts_lohi(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t b_hi,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 bd;\n\t"
      "mov.b64 bd, {%2, %3};\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], bd, %4, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 bit, 32 consecutive columns per thread. The load and its
// tcgen05.wait::ld sit in one asm statement, so the compiler cannot use the
// destination registers before the data has arrived.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// 64 consecutive columns per thread: two x32 loads and one wait in one asm statement.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&f)[64]) {
#define FA_R8(b) "=f"(f[b]), "=f"(f[b + 1]), "=f"(f[b + 2]), "=f"(f[b + 3]), "=f"(f[b + 4]), "=f"(f[b + 5]), \
                 "=f"(f[b + 6]), "=f"(f[b + 7])
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : FA_R8(0), FA_R8(8), FA_R8(16), FA_R8(24), FA_R8(32), FA_R8(40), FA_R8(48), FA_R8(56)
      : "r"(taddr), "r"(taddr + 32)
      : "memory");
#undef FA_R8
}

// 128 consecutive columns per thread: four x32 loads issued back to back and
// one tcgen05.wait::ld, all inside one asm statement (outputs valid after it).
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float (&f)[128]) {
#define FA_R8(b) "=f"(f[b]), "=f"(f[b + 1]), "=f"(f[b + 2]), "=f"(f[b + 3]), "=f"(f[b + 4]), "=f"(f[b + 5]), \
                 "=f"(f[b + 6]), "=f"(f[b + 7])
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%128];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%129];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,"
      "%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95}, [%130];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,"
      "%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%131];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : FA_R8(0), FA_R8(8), FA_R8(16), FA_R8(24), FA_R8(32), FA_R8(40), FA_R8(48), FA_R8(56), FA_R8(64),
        FA_R8(72), FA_R8(80), FA_R8(88), FA_R8(96), FA_R8(104), FA_R8(112), FA_R8(120)
      : "r"(taddr), "r"(taddr + 32), "r"(taddr + 64), "r"(taddr + 96)
      : "memory");
#undef FA_R8
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 16 consecutive columns per thread, load and wait in one asm statement.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// ------------------------------------------------------- smem descriptors
// tcgen05 shared-memory matrix descriptor (sm_100 format, version 1):
//   [0,14) start address >> 4, [16,30) leading byte offset >> 4,
//   [32,46) stride byte offset >> 4, [46,48) version = 1,
//   [49,52) base offset = 0 (atoms 1024-B aligned), [61,64) layout type.
constexpr uint64_t kLayoutSW128 = 2;

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes,
                                              uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= kLayoutSW128 << 61;
  return d;
}

// Instruction descriptor of kind::f16 with fp32 accumulation.
//   [4,6) c format (1 = f32), [7,10) a format, [10,13) b format
//   (0 = f16, 1 = bf16), [15] a major, [16] b major (0 = K, 1 = MN),
//   [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t m, uint32_t n, uint32_t ab_fmt,
                                                  uint32_t a_mn_major, uint32_t b_mn_major) {
  return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (a_mn_major << 15) | (b_mn_major << 16) |
         ((n >> 3) << 17) | ((m >> 4) << 24);
}

// Warpgroup register reallocation (all 128 threads of the warpgroup execute it).
template <uint32_t N>
__device__ __forceinline__ void reg_alloc_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void reg_alloc_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------- math
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Maximum of 128 values as a shallow tree of 3-input max instructions.
__device__ __forceinline__ float row_max128(const float (&s)[128]) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmax3f(s[i], s[i + 8], s[i + 16]);
#pragma unroll
  for (int k = 3; k < 15; k += 2)
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = fmax3f(m[i], s[i + 8 * k], s[i + 8 * k + 8]);
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmaxf(m[i], s[i + 120]);
  return fmax3f(fmax3f(m[0], m[1], m[2]), fmax3f(m[3], m[4], m[5]), fmaxf(m[6], m[7]));
}

// Maximum of 64 values as a shallow tree of 3-input max instructions.
__device__ __forceinline__ float row_max64(const float (&s)[64]) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmax3f(s[i], s[i + 8], s[i + 16]);
#pragma unroll
  for (int k = 3; k < 7; k += 2)
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = fmax3f(m[i], s[i + 8 * k], s[i + 8 * k + 8]);
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmaxf(m[i], s[i + 56]);
  return fmax3f(fmax3f(m[0], m[1], m[2]), fmax3f(m[3], m[4], m[5]), fmaxf(m[6], m[7]));
}

// 2^x for two values on the FMA/ALU pipes instead of MUFU.
// Method: Cody-Waite style range reduction x = n + f with n = round(x)
// (adding 1.5 * 2^23 rounds to an integer), f in [-1/2, 1/2], and a degree-3
// polynomial for 2^f whose coefficients were fitted for this build by the
// Remez exchange algorithm on the relative error over [-1/2, 1/2]
// (max relative error 7.5e-5, below the 2^-11 rounding of the fp16 P it
// feeds). The result is 2^n * p(f), formed by adding n to the exponent
// field. Inputs are clamped at -126 so the exponent never underflows.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kC0 = 0.99992807f, kC1 = 0.69326099f, kC2 = 0.24261112f, kC3 = 0.05517167f;
  constexpr float kRound = 12582912.f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 r = __fadd2_rn(x, make_float2(kRound, kRound));            // n in the low mantissa bits
  const float2 n = __fadd2_rn(r, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);              // x - n
  float2 p = __ffma2_rn(make_float2(kC3, kC3), f, make_float2(kC2, kC2));
  p = __ffma2_rn(p, f, make_float2(kC1, kC1));
  p = __ffma2_rn(p, f, make_float2(kC0, kC0));
  // (bits(r) << 23) == n << 23: the constant's low 9 bits are zero.
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(r.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(r.y) << 23)));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_bf162(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Rotate-half RoPE of 8 column pairs (x_i, x_{i+D/2}) (common.metal:150-167):
//   x_i' = x_i cos - x_{i+D/2} sin,  x_{i+D/2}' = x_i sin + x_{i+D/2} cos.
// The rounding steps are spelled out (no compiler-chosen contraction), so the
// result does not depend on how a kernel around it is compiled.
__device__ __forceinline__ void rope_rotate8(const float (&a)[8], const float (&b)[8], const float (&c)[8],
                                             const float (&s)[8], float (&ra)[8], float (&rb)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    ra[i] = __fmaf_rn(a[i], c[i], -__fmul_rn(b[i], s[i]));
    rb[i] = __fmaf_rn(a[i], s[i], __fmul_rn(b[i], c[i]));
  }
}

}  // namespace fa
