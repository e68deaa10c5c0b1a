// Device-side primitives for sm_100a: shared-memory barriers with bounded
// waits, TMA tile loads, and the tcgen05 (5th-generation tensor core) MMA,
// commit and tensor-memory operations, written as inline PTX.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace smm {

// Device error word bits (written with atomicOr into the per-call status).
enum : uint32_t {
  kDevErrTimeout = 1u << 0,
  kDevErrBounds = 1u << 1,  // debug builds: an index check caught an out-of-range read (skipped)
  // Which check fired (ORed with kDevErrBounds).
  kBoundsA = 1u << 16,       // structured left operand (packed triangle / Toeplitz generator)
  kBoundsB = 1u << 17,       // structured right operand
  kBoundsExpand = 1u << 18,  // packed-operand expansion
  // Which wait gave up (ORed with kDevErrTimeout).
  kWaitProducer = 1u << 8,   // producer waiting for a free stage
  kWaitMma = 1u << 9,        // MMA issuer waiting for a staged k-block
  kWaitTransform = 1u << 10, // transform warps waiting for TMA data
  kWaitEpilogue = 1u << 11,  // epilogue waiting for the accumulator
  kWaitDrain = 1u << 12,     // teardown drain
  kWaitProbe = 1u << 13,     // timeout probe
};

// Bounds-checked debug build (compiled with -DSMM_DEBUG_BOUNDS: the
// library's libsmm_debug.so).  Every computed offset into a structured
// operand is checked against the operand's element count; an offset outside
// it sets kDevErrBounds | where in the status word and the read is skipped
// (zero) instead of made.  In the normal build the checks compile away.
#ifdef SMM_DEBUG_BOUNDS
constexpr bool kDebugBounds = true;
#else
constexpr bool kDebugBounds = false;
#endif
__device__ __forceinline__ bool dbg_ok(long long off, long long limit, uint32_t* status, uint32_t where) {
  if constexpr (kDebugBounds) {
    if (off < 0 || off >= limit) {
      if (status) atomicOr(status, kDevErrBounds | where);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ float ld_chk(const float* __restrict__ src, long long off, long long limit,
                                        uint32_t* status, uint32_t where) {
  return dbg_ok(off, limit, status, where) ? __ldg(src + off) : 0.0f;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// The same with an explicit bound on how long the hardware may suspend the
// thread inside the try (ns): it resumes when the phase completes or when the
// hint elapses, whichever is first.  Without a hint the suspension bound is
// system-defined and can exceed a short wait limit.
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t bar_addr, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Shared state every role of a pipelined kernel consults while waiting: an
// abort flag in shared memory (set by whichever role gives up first, so the
// others stop waiting too), the wait limit, and the kernel's device status
// word in global memory.
struct WaitCtx {
  volatile int* abort_flag;  // shared memory
  uint32_t* status;          // global memory, may be null
  uint64_t limit_ns;
  uint32_t where;            // kWait* tag recorded on expiry
};

// Wait until the barrier phase with the given parity has completed.  Bounded:
// returns false (and raises the abort flag, records kDevErrTimeout) once
// limit_ns of wall time has passed, or as soon as another role aborted.
// Each try suspends the thread for at most limit/8 (between 100 ns and
// 20 us), so the limit, the abort flag and a completing phase are all seen
// promptly.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const WaitCtx& w) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t h = w.limit_ns / 8;
  const uint32_t hint = static_cast<uint32_t>(h < 100 ? 100 : (h > 20000 ? 20000 : h));
  while (true) {
    if (mbar_try_wait_hint(a, parity, hint)) return true;
    if (*w.abort_flag) return false;
    if (globaltimer_ns() - t0 > w.limit_ns) {
      *w.abort_flag = 1;
      if (w.status) atomicOr(w.status, kDevErrTimeout | w.where);
      return false;
    }
  }
}

// ---------------------------------------------------------------- fences
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor load global -> shared, completing on `bar` with the
// transaction byte count.  c0 is the innermost (contiguous) coordinate.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// ---------------------------------------------------------------- cp.async
// 4-byte asynchronous copy global -> shared; src_bytes = 0 writes a zero
// without reading global memory (the source address is then unused).
__device__ __forceinline__ void cp_async_4(uint32_t smem_dst, const float* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_dst), "l"(src), "r"(src_bytes)
               : "memory");
}
// 16-byte asynchronous copy global -> shared, both 16-byte aligned, through L1.
__device__ __forceinline__ void cp_async_16(uint32_t smem_dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(smem_dst), "l"(src) : "memory");
}
// Arrive on `bar` once every cp.async this thread issued so far has landed.
// The arrival is not pre-counted (.noinc): the barrier's expected count
// includes it.
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------------- tcgen05
// Tensor-memory allocation by one full warp; the TMEM base address is written
// to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// tcgen05.mma with the shared-memory descriptors given as 32-bit halves (the
// issue loop advances only the start-address field in the low word, with
// 32-bit adds).  PAIR selects .cta_group::2, BF16 kind::f16, else kind::tf32.
template <bool PAIR, bool BF16>
__device__ __forceinline__ void umma_lohi(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo, uint32_t b_hi,
                                          uint32_t idesc, uint32_t accumulate) {
  if constexpr (PAIR && BF16) {
    asm volatile(
        "{\n\t.reg .b64 da, db;\n\t.reg .pred p;\n\t"
        "mov.b64 da, {%1, %2};\n\tmov.b64 db, {%3, %4};\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], da, db, %5, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (PAIR) {
    asm volatile(
        "{\n\t.reg .b64 da, db;\n\t.reg .pred p;\n\t"
        "mov.b64 da, {%1, %2};\n\tmov.b64 db, {%3, %4};\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], da, db, %5, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (BF16) {
    asm volatile(
        "{\n\t.reg .b64 da, db;\n\t.reg .pred p;\n\t"
        "mov.b64 da, {%1, %2};\n\tmov.b64 db, {%3, %4};\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .b64 da, db;\n\t.reg .pred p;\n\t"
        "mov.b64 da, {%1, %2};\n\tmov.b64 db, {%3, %4};\n\t"
        "setp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], da, db, %5, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Commit to an mbarrier given by its (shared::cta or shared::cluster) address.
template <bool PAIR>
__device__ __forceinline__ void umma_commit_addr(uint32_t bar_addr) {
  if constexpr (PAIR)
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_addr)
                 : "memory");
  else
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_addr)
                 : "memory");
}

// Arrive once on `bar` when every tcgen05.mma this thread issued so far has
// completed (and its shared-memory operands may be overwritten).
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns of tensor memory into registers
// (lane i of the warp gets TMEM lane (taddr.lane + i)).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Registers into 32 lanes x 16 consecutive 32-bit columns of tensor memory.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- CTA pairs
// A pair is a cluster of two CTAs on neighbouring SMs.  One tcgen05.mma with
// .cta_group::2 (issued by the even CTA) computes a 256 x N tile: CTA v
// supplies rows [128v, 128v+128) of A and columns [v N/2, (v+1) N/2) of B from
// its own shared memory (same offsets in both CTAs), and receives rows
// [128v, 128v+128) of D in its own tensor memory.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Shared::cluster address of the variable at shared::cta address `a` in CTA
// `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t a, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(rank));
  return d;
}
// Arrive on an mbarrier of any CTA of the cluster (default semantics:
// release at CTA scope, so no cluster-wide memory fence per arrival; the
// shared-memory tiles it hands over were already made visible to the tensor
// core by fence.proxy.async).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 16-byte store to shared memory of any CTA of the cluster (address from
// mapa_shared).
__device__ __forceinline__ void st_cluster_v4(uint32_t cluster_addr, uint32_t a, uint32_t b, uint32_t c,
                                              uint32_t d) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
// Every thread of both CTAs; orders each CTA's prior writes (barrier
// initialisation, tensor-memory allocation) before the other's later reads.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Pair-wide tensor-memory allocation: the same warp of both CTAs issues it,
// with the same destination offset.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrive once on the mbarrier at shared::cluster address `cluster_addr` (in
// either CTA of the pair) when every pair MMA this thread issued so far has
// completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
               : "memory");
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor (tcgen05 format): start address, leading
// and stride byte offsets (all >> 4), version 1, layout/swizzle type
// (0 none, 2 = 128B, 4 = 64B, 6 = 32B swizzle).
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                                   uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// Layout types of the matrix descriptor.  kLayoutSw128Base32 is the 128-byte
// swizzle with 32-byte atoms (address bits [5,7) ^= bits [7,9)), the layout
// an MN-major 32-bit (tf32) operand must use; TMA writes it with
// CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B.
enum : uint32_t { kLayoutSw128Base32 = 1, kLayoutSw128 = 2, kLayoutSw64 = 4, kLayoutSw32 = 6 };
enum : uint32_t { kFmtF16 = 0, kFmtBF16 = 1, kFmtTF32 = 2 };

// Instruction descriptor for kind::tf32 / kind::f16 with fp32 accumulation.
// a_mn / b_mn select MN-major (1) instead of K-major (0) operands.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t ab_fmt, uint32_t M, uint32_t N, uint32_t a_mn,
                                                  uint32_t b_mn) {
  return (1u << 4)                // D format: f32
         | (ab_fmt << 7)          // A format
         | (ab_fmt << 10)         // B format
         | (a_mn << 15)           // A major
         | (b_mn << 16)           // B major
         | ((N >> 3) << 17)       // N / 8
         | ((M >> 4) << 24);      // M / 16
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a K-major tile whose
// rows are `row_bytes` long (64 or 128) and swizzled the way TMA's
// CU_TENSOR_MAP_SWIZZLE_64B / _128B modes place them (the tile base being
// aligned to 1024 bytes).
__device__ __forceinline__ uint32_t swz_offset(uint32_t row, uint32_t chunk, uint32_t row_bytes) {
  if (row_bytes == 128) return row * 128u + ((chunk ^ (row & 7u)) << 4);
  // 64-byte rows: address bits [4,5] ^= bits [7,8]
  return row * 64u + ((chunk ^ ((row >> 1) & 3u)) << 4);
}

// tf32 split: hi keeps the 19 most significant bits (sign, exponent, 10
// mantissa bits), lo = x - hi is exact in fp32.
__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

}  // namespace smm
