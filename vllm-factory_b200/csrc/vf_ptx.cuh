// Inline-PTX building blocks for the sm_100a attention kernels: mbarriers with
// bounded waits, TMA tile loads (no cluster multicast anywhere), tcgen05 TMEM
// allocation, UMMA issue/commit and TMEM <-> register moves.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace vf {

// Device-wide error word of this translation unit.  Kernels OR error bits into it (a
// bounded wait that ran out, an index that failed a check); the host takes it with
// take_error_word() (vf_device_error() gathers the words of every kernel file).
static __device__ unsigned int g_vf_error;
static __device__ unsigned int g_vf_error_taken;

// Reads the word and, with `clear`, zeroes it in the same atomic operation, so a bit that a
// kernel on another stream sets meanwhile is either taken now or stays for the next call.
static __global__ void take_error_word_kernel(int clear) {
  g_vf_error_taken = clear ? atomicExch(&g_vf_error, 0u) : atomicOr(&g_vf_error, 0u);
}

enum : unsigned int {
  kErrWaitTimeout = 1u << 0,   // an mbarrier wait exceeded its cycle budget
  kErrBadIndex    = 1u << 1,   // a gather index failed its bounds check (skipped)
  kErrBadInput    = 1u << 2,   // an input broke a documented limit (e.g. a sequence longer than max_seqlen)
};

// A wait that has spun this many SM cycles (~1 s at 1.9 GHz) gives up and flags an error.
constexpr long long kWaitCycles = 2000000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// As above, but the thread may sleep up to `suspend_ns` (it wakes when the phase
// completes), so waiting warps do not take issue slots from working ones.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t suspend_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok) : "r"(bar), "r"(parity), "r"(suspend_ns) : "memory");
  return ok != 0;
}
constexpr uint32_t kSuspendNs = 20000;   // 20 us per sleep; the cycle bound still applies

// Waits for the phase with the given parity to complete.  Every wait is bounded: after
// kWaitCycles it sets the CTA abort flag and the global error word and returns false.  A
// wait also returns false as soon as another thread of the CTA has set the abort flag,
// so one stalled role cannot leave the others spinning.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          long long limit_cycles = kWaitCycles) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_sleep(a, parity, kSuspendNs)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > limit_cycles) {
      *abort_flag = 1;
      atomicOr(&g_vf_error, kErrWaitTimeout);
      return false;
    }
  }
}

// Time-bounded wait that ignores the abort flag (teardown: drain outstanding copies).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  const long long t0 = clock64();
  while (!mbar_try_wait(a, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      atomicOr(&g_vf_error, kErrWaitTimeout);
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------- TMA (tiled, no multicast)
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];"
      :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)),
         "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];"
      :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];"
      :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Tiled bulk store shared -> global (async proxy), tracked by bulk groups.  Elements
// outside the tensor's extent are not written.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];"
               :: "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
               :: "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(c0), "r"(c1) : "memory");
}
// The thread's committed bulk stores other than the newest N have finished reading shared memory.
template <int N> __device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" :: "n"(N) : "memory");
}
// Untiled bulk copy shared -> global (async proxy), bulk-group completion; addresses
// 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_copy_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
               :: "l"(reinterpret_cast<uint64_t>(dst)), "r"(smem_u32(src)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The thread's committed bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// The thread's committed bulk stores have completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's generic-proxy shared-memory writes before later async-proxy reads.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------- tcgen05: TMEM management
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05: UMMA
// Arrives once on `bar` when every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_u32(bar)) : "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc)^T
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
      :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// D(tmem) (+)= A(tmem) * B(smem desc)
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n"
      :: "r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

// Shared-memory matrix descriptor for a tile written by TMA with 128-byte swizzling.
// Rows are 128 bytes; 8-row core groups are `sbo` bytes apart.  Field layout: start
// address >> 4 in bits [0,14), leading byte offset >> 4 in [16,30), stride byte offset >> 4
// in [32,46), version 1 in [46,48), swizzle mode in [61,64) (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// General shared-memory matrix descriptor: `layout` is the tcgen05 swizzle code in bits
// [61,64): 0 = none, 2 = 128-byte, 4 = 64-byte, 6 = 32-byte swizzle.  For a K-major operand
// `sbo` is the distance between 8-row groups; for an MN-major swizzled operand `lbo` is the
// distance between the MN blocks one swizzle row wide and `sbo` between 8-row K groups.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}
constexpr uint32_t kLayoutSw128 = 2, kLayoutSw64 = 4;

// Instruction descriptor for kind::f16 with an fp32 accumulator.
//   ab_fmt: 0 = fp16, 1 = bf16;  a_mn / b_mn: operand is MN-major (1) or K-major (0).
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t ab_fmt, uint32_t M, uint32_t N,
                                                 uint32_t a_mn, uint32_t b_mn) {
  return (1u << 4)                 // D format fp32
       | (ab_fmt << 7) | (ab_fmt << 10)
       | (a_mn << 15) | (b_mn << 16)
       | ((N >> 3) << 17)
       | ((M >> 4) << 24);
}

// ---------------------------------------------------------------- tcgen05: TMEM <-> registers
// 32x32b shape: thread t of the warp reads/writes TMEM lane (32 * (warp % 4) + t), N
// consecutive 32-bit columns starting at the address's column.  The wait is part of the
// same asm statement so no consumer of the registers can be scheduled before it.
__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
               "tcgen05.wait::ld.sync.aligned;\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
               : "r"(taddr) : "memory");
}

__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
               "tcgen05.wait::ld.sync.aligned;\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
               : "r"(taddr) : "memory");
}

__device__ __forceinline__ void tmem_ld_x64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n"
               "tcgen05.wait::ld.sync.aligned;\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
               : "r"(taddr) : "memory");
}

__device__ __forceinline__ void tmem_ld_x128(uint32_t taddr, uint32_t (&r)[128]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];\n"
               "tcgen05.wait::ld.sync.aligned;\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
               : "r"(taddr) : "memory");
}

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n"
               "tcgen05.wait::st.sync.aligned;\n"
               :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]) : "memory");
}

__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n"
               "tcgen05.wait::st.sync.aligned;\n"
               :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]) : "memory");
}

__device__ __forceinline__ void tmem_st_x64(uint32_t taddr, const uint32_t (&r)[64]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64};\n"
               "tcgen05.wait::st.sync.aligned;\n"
               :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]), "r"(r[32]), "r"(r[33]), "r"(r[34]), "r"(r[35]), "r"(r[36]), "r"(r[37]), "r"(r[38]), "r"(r[39]), "r"(r[40]), "r"(r[41]), "r"(r[42]), "r"(r[43]), "r"(r[44]), "r"(r[45]), "r"(r[46]), "r"(r[47]), "r"(r[48]), "r"(r[49]), "r"(r[50]), "r"(r[51]), "r"(r[52]), "r"(r[53]), "r"(r[54]), "r"(r[55]), "r"(r[56]), "r"(r[57]), "r"(r[58]), "r"(r[59]), "r"(r[60]), "r"(r[61]), "r"(r[62]), "r"(r[63]) : "memory");
}

// Loads 64 consecutive fp32 columns of this thread's TMEM lane into x[32] (pairs).
__device__ __forceinline__ void tmem_ld_x64_f2(uint32_t taddr, float2 (&x)[32]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n"
               "tcgen05.wait::ld.sync.aligned;\n"
               : "=f"(x[0].x), "=f"(x[0].y), "=f"(x[1].x), "=f"(x[1].y), "=f"(x[2].x), "=f"(x[2].y), "=f"(x[3].x), "=f"(x[3].y), "=f"(x[4].x), "=f"(x[4].y), "=f"(x[5].x), "=f"(x[5].y), "=f"(x[6].x), "=f"(x[6].y), "=f"(x[7].x), "=f"(x[7].y), "=f"(x[8].x), "=f"(x[8].y), "=f"(x[9].x), "=f"(x[9].y), "=f"(x[10].x), "=f"(x[10].y), "=f"(x[11].x), "=f"(x[11].y), "=f"(x[12].x), "=f"(x[12].y), "=f"(x[13].x), "=f"(x[13].y), "=f"(x[14].x), "=f"(x[14].y), "=f"(x[15].x), "=f"(x[15].y), "=f"(x[16].x), "=f"(x[16].y), "=f"(x[17].x), "=f"(x[17].y), "=f"(x[18].x), "=f"(x[18].y), "=f"(x[19].x), "=f"(x[19].y), "=f"(x[20].x), "=f"(x[20].y), "=f"(x[21].x), "=f"(x[21].y), "=f"(x[22].x), "=f"(x[22].y), "=f"(x[23].x), "=f"(x[23].y), "=f"(x[24].x), "=f"(x[24].y), "=f"(x[25].x), "=f"(x[25].y), "=f"(x[26].x), "=f"(x[26].y), "=f"(x[27].x), "=f"(x[27].y), "=f"(x[28].x), "=f"(x[28].y), "=f"(x[29].x), "=f"(x[29].y), "=f"(x[30].x), "=f"(x[30].y), "=f"(x[31].x), "=f"(x[31].y)
               : "r"(taddr) : "memory");
}

// Loads 128 consecutive fp32 columns of this thread's TMEM lane into x[64] (pairs) and
// waits for them, in one asm statement.
__device__ __forceinline__ void tmem_ld_x128_f2(uint32_t taddr, float2 (&x)[64]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];\n"
               "tcgen05.wait::ld.sync.aligned;\n"
               : "=f"(x[0].x), "=f"(x[0].y), "=f"(x[1].x), "=f"(x[1].y), "=f"(x[2].x), "=f"(x[2].y), "=f"(x[3].x), "=f"(x[3].y), "=f"(x[4].x), "=f"(x[4].y), "=f"(x[5].x), "=f"(x[5].y), "=f"(x[6].x), "=f"(x[6].y), "=f"(x[7].x), "=f"(x[7].y), "=f"(x[8].x), "=f"(x[8].y), "=f"(x[9].x), "=f"(x[9].y), "=f"(x[10].x), "=f"(x[10].y), "=f"(x[11].x), "=f"(x[11].y), "=f"(x[12].x), "=f"(x[12].y), "=f"(x[13].x), "=f"(x[13].y), "=f"(x[14].x), "=f"(x[14].y), "=f"(x[15].x), "=f"(x[15].y), "=f"(x[16].x), "=f"(x[16].y), "=f"(x[17].x), "=f"(x[17].y), "=f"(x[18].x), "=f"(x[18].y), "=f"(x[19].x), "=f"(x[19].y), "=f"(x[20].x), "=f"(x[20].y), "=f"(x[21].x), "=f"(x[21].y), "=f"(x[22].x), "=f"(x[22].y), "=f"(x[23].x), "=f"(x[23].y), "=f"(x[24].x), "=f"(x[24].y), "=f"(x[25].x), "=f"(x[25].y), "=f"(x[26].x), "=f"(x[26].y), "=f"(x[27].x), "=f"(x[27].y), "=f"(x[28].x), "=f"(x[28].y), "=f"(x[29].x), "=f"(x[29].y), "=f"(x[30].x), "=f"(x[30].y), "=f"(x[31].x), "=f"(x[31].y), "=f"(x[32].x), "=f"(x[32].y), "=f"(x[33].x), "=f"(x[33].y), "=f"(x[34].x), "=f"(x[34].y), "=f"(x[35].x), "=f"(x[35].y), "=f"(x[36].x), "=f"(x[36].y), "=f"(x[37].x), "=f"(x[37].y), "=f"(x[38].x), "=f"(x[38].y), "=f"(x[39].x), "=f"(x[39].y), "=f"(x[40].x), "=f"(x[40].y), "=f"(x[41].x), "=f"(x[41].y), "=f"(x[42].x), "=f"(x[42].y), "=f"(x[43].x), "=f"(x[43].y), "=f"(x[44].x), "=f"(x[44].y), "=f"(x[45].x), "=f"(x[45].y), "=f"(x[46].x), "=f"(x[46].y), "=f"(x[47].x), "=f"(x[47].y), "=f"(x[48].x), "=f"(x[48].y), "=f"(x[49].x), "=f"(x[49].y), "=f"(x[50].x), "=f"(x[50].y), "=f"(x[51].x), "=f"(x[51].y), "=f"(x[52].x), "=f"(x[52].y), "=f"(x[53].x), "=f"(x[53].y), "=f"(x[54].x), "=f"(x[54].y), "=f"(x[55].x), "=f"(x[55].y), "=f"(x[56].x), "=f"(x[56].y), "=f"(x[57].x), "=f"(x[57].y), "=f"(x[58].x), "=f"(x[58].y), "=f"(x[59].x), "=f"(x[59].y), "=f"(x[60].x), "=f"(x[60].y), "=f"(x[61].x), "=f"(x[61].y), "=f"(x[62].x), "=f"(x[62].y), "=f"(x[63].x), "=f"(x[63].y)
               : "r"(taddr) : "memory");
}

// 128 columns as two x64 loads and one wait: each tcgen05.ld names at most 64
// destination registers, so the instruction also fits a 128-register launch bound.
__device__ __forceinline__ void tmem_ld_2x64_f2(uint32_t taddr, float2 (&x)[64]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%128];\n"
               "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%129];\n"
               "tcgen05.wait::ld.sync.aligned;\n"
               : "=f"(x[0].x), "=f"(x[0].y), "=f"(x[1].x), "=f"(x[1].y), "=f"(x[2].x), "=f"(x[2].y), "=f"(x[3].x), "=f"(x[3].y), "=f"(x[4].x), "=f"(x[4].y), "=f"(x[5].x), "=f"(x[5].y), "=f"(x[6].x), "=f"(x[6].y), "=f"(x[7].x), "=f"(x[7].y), "=f"(x[8].x), "=f"(x[8].y), "=f"(x[9].x), "=f"(x[9].y), "=f"(x[10].x), "=f"(x[10].y), "=f"(x[11].x), "=f"(x[11].y), "=f"(x[12].x), "=f"(x[12].y), "=f"(x[13].x), "=f"(x[13].y), "=f"(x[14].x), "=f"(x[14].y), "=f"(x[15].x), "=f"(x[15].y), "=f"(x[16].x), "=f"(x[16].y), "=f"(x[17].x), "=f"(x[17].y), "=f"(x[18].x), "=f"(x[18].y), "=f"(x[19].x), "=f"(x[19].y), "=f"(x[20].x), "=f"(x[20].y), "=f"(x[21].x), "=f"(x[21].y), "=f"(x[22].x), "=f"(x[22].y), "=f"(x[23].x), "=f"(x[23].y), "=f"(x[24].x), "=f"(x[24].y), "=f"(x[25].x), "=f"(x[25].y), "=f"(x[26].x), "=f"(x[26].y), "=f"(x[27].x), "=f"(x[27].y), "=f"(x[28].x), "=f"(x[28].y), "=f"(x[29].x), "=f"(x[29].y), "=f"(x[30].x), "=f"(x[30].y), "=f"(x[31].x), "=f"(x[31].y), "=f"(x[32].x), "=f"(x[32].y), "=f"(x[33].x), "=f"(x[33].y), "=f"(x[34].x), "=f"(x[34].y), "=f"(x[35].x), "=f"(x[35].y), "=f"(x[36].x), "=f"(x[36].y), "=f"(x[37].x), "=f"(x[37].y), "=f"(x[38].x), "=f"(x[38].y), "=f"(x[39].x), "=f"(x[39].y), "=f"(x[40].x), "=f"(x[40].y), "=f"(x[41].x), "=f"(x[41].y), "=f"(x[42].x), "=f"(x[42].y), "=f"(x[43].x), "=f"(x[43].y), "=f"(x[44].x), "=f"(x[44].y), "=f"(x[45].x), "=f"(x[45].y), "=f"(x[46].x), "=f"(x[46].y), "=f"(x[47].x), "=f"(x[47].y), "=f"(x[48].x), "=f"(x[48].y), "=f"(x[49].x), "=f"(x[49].y), "=f"(x[50].x), "=f"(x[50].y), "=f"(x[51].x), "=f"(x[51].y), "=f"(x[52].x), "=f"(x[52].y), "=f"(x[53].x), "=f"(x[53].y), "=f"(x[54].x), "=f"(x[54].y), "=f"(x[55].x), "=f"(x[55].y), "=f"(x[56].x), "=f"(x[56].y), "=f"(x[57].x), "=f"(x[57].y), "=f"(x[58].x), "=f"(x[58].y), "=f"(x[59].x), "=f"(x[59].y), "=f"(x[60].x), "=f"(x[60].y), "=f"(x[61].x), "=f"(x[61].y), "=f"(x[62].x), "=f"(x[62].y), "=f"(x[63].x), "=f"(x[63].y)
               : "r"(taddr), "r"(taddr + 64u) : "memory");
}

// Five 16-column loads at taddr, taddr + 16, ..., taddr + 64 into r[0..80) and one
// 2-column load at taddr2 into e[0..2), then one wait: a single TMEM round trip for 82
// columns of this thread's lane.
__device__ __forceinline__ void tmem_ld_5x16_x2(uint32_t taddr, uint32_t taddr2, uint32_t (&r)[80], uint32_t (&e)[2]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%82];\n"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%83];\n"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47}, [%84];\n"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%85];\n"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79}, [%86];\n"
      "tcgen05.ld.sync.aligned.32x32b.x2.b32 {%80, %81}, [%87];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(e[0]), "=r"(e[1])
      : "r"(taddr), "r"(taddr + 16u), "r"(taddr + 32u), "r"(taddr + 48u), "r"(taddr + 64u), "r"(taddr2)
      : "memory");
}

// tcgen05.ld of 16 columns without waiting: the registers are written asynchronously and
// must not be read before tmem_wait_ld_regs() on them.
__device__ __forceinline__ void tmem_ld_x16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
               : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tmem_ld_x2_nowait(uint32_t taddr, uint32_t (&r)[2]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];\n" : "=r"(r[0]), "=r"(r[1]) : "r"(taddr) : "memory");
}
// Waits for this thread's TMEM loads; the registers are named as read and written here so
// that no use of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :: "memory");
}
__device__ __forceinline__ void tmem_wait_ld_regs2(uint32_t (&r)[16], uint32_t (&e)[2]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(e[0]), "+r"(e[1])
               :: "memory");
}

// 16 columns at taddr and 2 at taddr2 (e.g. the two after the group), without waiting.
__device__ __forceinline__ void tmem_ld_x16_x2_nowait(uint32_t taddr, uint32_t taddr2, uint32_t (&r)[16], uint32_t (&e)[2]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%18];\n"
               "tcgen05.ld.sync.aligned.32x32b.x2.b32 {%16,%17}, [%19];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                 "=r"(e[0]), "=r"(e[1])
               : "r"(taddr), "r"(taddr2) : "memory");
}

// tcgen05.st of 16 columns without waiting; the caller issues tmem_wait_st() before the
// data is consumed.  The source registers are read when the instruction issues.
__device__ __forceinline__ void tmem_st_x16_nowait(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n"
               :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
                  "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
               : "memory");
}
__device__ __forceinline__ void tmem_st_x32_nowait(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n"
               :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]) : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- math helpers
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// fp32 pair -> f16x2 with saturation to the finite range (lo in bits 0-15).
__device__ __forceinline__ uint32_t pack_f16x2_sat(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// Byte permute of the pair {b:a} (a = bytes 0-3, b = bytes 4-7); `sel` may differ per lane.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
__device__ __forceinline__ void st_shared_u32(uint32_t saddr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" :: "r"(saddr), "r"(v) : "memory");
}

// Per-warpgroup register budget moves (all warps of a warpgroup execute the same one).
template <uint32_t N> __device__ __forceinline__ void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" :: "n"(N));
}
template <uint32_t N> __device__ __forceinline__ void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" :: "n"(N));
}

// 2^y for a pair on the FMA pipe (offloads the MUFU unit, whose ex2 throughput caps
// attention with 64-wide heads).  Method: y clamped to >= -125; y = j + f with
// j = round(y) obtained from y + 1.5*2^23 (round-to-nearest in the float adder) and
// f in [-0.5, 0.5]; 2^f by a degree-3 polynomial whose coefficients are a minimax fit of
// the relative error over [-0.5, 0.5] (max relative error 7.5e-5, far below bf16/fp16
// resolution); 2^j applied by adding j to the exponent field: the low mantissa bits of
// y + 1.5*2^23 hold j, so (bits << 23) is j * 2^23 modulo 2^32.
__device__ __forceinline__ float2 exp2_poly2(float2 y) {
  constexpr float kRound = 12582912.0f;   // 1.5 * 2^23
  constexpr float c0 = 0.99992806f, c1 = 0.69326097f, c2 = 0.24261113f, c3 = 0.05517167f;
  y.x = fmaxf(y.x, -125.0f);
  y.y = fmaxf(y.y, -125.0f);
  const float2 t = __fadd2_rn(y, make_float2(kRound, kRound));
  const float2 j = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(j, make_float2(-1.0f, -1.0f), y);
  float2 q = __ffma2_rn(make_float2(c3, c3), f, make_float2(c2, c2));
  q = __ffma2_rn(q, f, make_float2(c1, c1));
  q = __ffma2_rn(q, f, make_float2(c0, c0));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// 2^x for two packed 16-bit values (MUFU, two results per lane and instruction).
__device__ __forceinline__ uint32_t ex2_bf16x2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.ftz.bf16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t ex2_f16x2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
// acc + lo16(p) and acc + hi16(p) for a packed bf16 pair, accumulated in fp32.
__device__ __forceinline__ void add_bf16x2_f32(float& acc_lo, float& acc_hi, uint32_t p) {
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "add.rn.f32.bf16 %0, lo, %0;\n\tadd.rn.f32.bf16 %1, hi, %1;\n\t}\n"
      : "+f"(acc_lo), "+f"(acc_hi) : "r"(p));
}
__device__ __forceinline__ void add_f16x2_f32(float& acc_lo, float& acc_hi, uint32_t p) {
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "add.rn.f32.f16 %0, lo, %0;\n\tadd.rn.f32.f16 %1, hi, %1;\n\t}\n"
      : "+f"(acc_lo), "+f"(acc_hi) : "r"(p));
}

// Named barrier over `nthreads` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}
// Named barrier over `nthreads` threads that also returns whether `pred` held on any of them
// (a decision every participating thread takes alike).
__device__ __forceinline__ bool named_bar_any(uint32_t id, uint32_t nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %3, 0;\n\t"
      "bar.red.or.pred p, %1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(r) : "r"(id), "r"(nthreads), "r"(pred ? 1u : 0u) : "memory");
  return r != 0;
}
// Arrives on a named barrier without waiting (the producer side of a hand-over).
__device__ __forceinline__ void named_bar_arrive(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.arrive %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

// Host side of take_error_word_kernel: one launch on the legacy default stream and a read
// of the result.  Returns the cudaError_t of the first failing call.
static inline cudaError_t take_error_word(bool clear, unsigned int* word) {
  take_error_word_kernel<<<1, 1, 0, 0>>>(clear ? 1 : 0);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return cudaMemcpyFromSymbol(word, g_vf_error_taken, sizeof(unsigned int));
}

}  // namespace vf
