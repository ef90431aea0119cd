// tc_common.cuh -- sm_100a building blocks: mbarriers with bounded waits,
// TMA tile loads, UMMA shared-memory / instruction descriptors, tcgen05 MMA,
// commit, TMEM allocation and loads.  Inline PTX, no library.
//
// Every wait is bounded in wall-clock time (%globaltimer): past the limit the
// waiter records an error code in the kernel's error word, raises the CTA's
// abort flag and returns, so a kernel whose partner never arrives ends with
// an error status instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include "common.cuh"

namespace zb {
namespace tc {

enum ErrCode : int {
    kErrFullWait = 0x54430001,    // producer data never arrived
    kErrEmptyWait = 0x54430002,   // consumer never released a stage
    kErrAccWait = 0x54430003,     // accumulator handshake timed out
    kErrDrain = 0x54430004,       // final drain of in-flight work timed out
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Every wait in these kernels is microseconds long when the partner is alive;
// two seconds of wall clock means it never will be.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr uint64_t kDrainLimitNs = 1000000000ull;

// Bounded wait for the phase with the given parity to complete.  Returns
// false (after recording `code`) when the time limit runs out or *abort is set.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                          int *err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0u) {
            if (*abort) return false;
            if (global_ns() - t0 > kWaitLimitNs) break;
        }
    }
    *abort = 1;
    if (err) atomicCAS(err, 0, code);
    return false;
}

// Bounded wait that ignores the abort flag: used to drain copies and MMAs
// already in flight before a kernel that aborted releases its resources.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t *bar, uint32_t parity) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && global_ns() - t0 > kDrainLimitNs) return false;
    }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1,
                                            int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1,
                                            int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}

// Tiled 2D TMA store shared -> global (no multicast); coordinates must be >= 0.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(c0),
                 "r"(c1), "r"(smem_u32(src))
                 : "memory");
}

// Tiled TMA store shared -> global (no multicast); coordinates must be >= 0.
// Out-of-range box elements are not written.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, const void *src, int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(map), "r"(c0),
        "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(src))
        : "memory");
}

// Untiled bulk copy shared -> global (no multicast): both addresses 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_store(void *gdst, const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(src)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until at most N committed bulk groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until all committed bulk groups of this thread are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Makes this thread's generic-proxy shared-memory writes visible to the async proxy (TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor (tcgen05 format): start address, leading
// and stride byte offsets (all >> 4), version 1, swizzle mode in bits 61-63.
// kSw128B32: the 128-byte swizzle over 32-byte atoms (4 rows of 128 B per atom), the
// only shared-memory layout of an MN-major operand of 32-bit elements (tf32).
enum Swizzle : uint32_t { kSwNone = 0, kSw128B32 = 1, kSw128 = 2, kSw64 = 4, kSw32 = 6 };

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, Swizzle sw) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;   // descriptor version for tcgen05
    d |= (uint64_t)sw << 61;
    return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 accumulation.
// a_mn / b_mn: operand is MN-major (else K-major).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
    return (1u << 4)                      // D format: f32
           | (1u << 7)                    // A format: bf16
           | (1u << 10)                   // B format: bf16
           | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}

// The same MMA with the A operand kept in the tensor core's collector buffer:
// OP 0 (fill) reads A from shared memory and keeps it, OP 1 (use) takes A from
// the buffer instead of shared memory, OP 2 (lastuse) takes it and releases
// the buffer.  For a run of MMAs that share one A (same descriptor), issued
// back to back by one thread.
template <int OP>
__device__ __forceinline__ void mma_bf16_ca(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            bool accumulate) {
    static_assert(OP >= 0 && OP <= 2, "collector op");
    if constexpr (OP == 0)
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16.collector::a::fill [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
            : "memory");
    else if constexpr (OP == 1)
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16.collector::a::use [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
            : "memory");
    else
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16.collector::a::lastuse [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
            : "memory");
}

// Arrives on `bar` once all previously issued MMAs of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Whole-warp TMEM allocation; the base address lands in *slot (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives
// row (lane base + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// relu(a + ba), relu(b + bb) rounded to bf16 and packed, a in the low half:
// one packed fp32 add (each lane rounded like a scalar add) and one
// conversion whose .relu clamps negative results to zero, which equals
// rounding relu(x) since rounding is monotonic and keeps zero.
__device__ __forceinline__ uint32_t bias_relu_bf16x2(float a, float b, float ba, float bb) {
    uint64_t x, y, s;
    asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a), "f"(b));
    asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(ba), "f"(bb));
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(s) : "l"(x), "l"(y));
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(s));
    uint32_t d;
    asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

// relu(a), relu(b) rounded to bf16 and packed, a in the low half.
__device__ __forceinline__ uint32_t relu_bf16x2(float a, float b) {
    uint32_t d;
    asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(b), "f"(a));
    return d;
}

// One step of a running 2x2 max-pool over bf16x2 words: where the candidate c
// is strictly greater (the first maximum wins ties), the lane's position
// becomes q; best becomes the lane-wise maximum.
__device__ __forceinline__ void pool_step_bf16x2(uint32_t &best, uint32_t &pos, uint32_t c, uint32_t q) {
    const __nv_bfloat162 cb = *reinterpret_cast<const __nv_bfloat162 *>(&c);
    __nv_bfloat162 bb = *reinterpret_cast<const __nv_bfloat162 *>(&best);
    const uint32_t m = __hgt2_mask(cb, bb);
    bb = __hmax2(bb, cb);
    best = *reinterpret_cast<const uint32_t *>(&bb);
    pos = (pos & ~m) | (q * 0x00010001u & m);
}

// Pool codes of two bf16x2 words of ReLU outputs: per channel a byte
// pos | 4 when the maximum is positive (non-zero magnitude bits), packed in
// channel order.
__device__ __forceinline__ uint32_t pool_codes(uint32_t best0, uint32_t pos0, uint32_t best1, uint32_t pos1) {
    const uint32_t nz0 = (((best0 & 0x7FFF7FFFu) + 0x7FFF7FFFu) & 0x80008000u) >> 13;
    const uint32_t nz1 = (((best1 & 0x7FFF7FFFu) + 0x7FFF7FFFu) & 0x80008000u) >> 13;
    return __byte_perm(pos0 | nz0, pos1 | nz1, 0x6420);
}

// Max-unpool of 8 channels: the lanes of pv whose code (a nibble of sel_lo for
// channels 0-3, sel_hi for 4-7; codes 0..7) selects a 0xFF byte of the table
// (0, tab), zero elsewhere.  tab = 0xFF << 8q keeps the channels routed to
// window position q (code 4 | q); tab = ~0 keeps every routed channel.
__device__ __forceinline__ uint4 unpool_select(uint4 pv, uint32_t sel_lo, uint32_t sel_hi, uint32_t tab) {
    const uint32_t m_lo = __byte_perm(0u, tab, sel_lo), m_hi = __byte_perm(0u, tab, sel_hi);
    return make_uint4(pv.x & __byte_perm(m_lo, 0u, 0x1100), pv.y & __byte_perm(m_lo, 0u, 0x3322),
                      pv.z & __byte_perm(m_hi, 0u, 0x1100), pv.w & __byte_perm(m_hi, 0u, 0x3322));
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
        "elect.sync rx|px, 0xffffffff;\n\t"
        "selp.b32 %0, 1, 0, px;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// ---------------------------------------------------------------- host
// Encodes a tiled TMA descriptor for a bf16 tensor (dims innermost first;
// strides in bytes for dims 1..rank-1).  Returns 0 on success.
int make_tmap_bf16(CUtensorMap *map, const void *base, int rank, const uint64_t *dims, const uint64_t *strides,
                   const uint32_t *box, Swizzle sw);
// The same for an fp32 tensor, and for any element type.
int make_tmap_f32(CUtensorMap *map, const void *base, int rank, const uint64_t *dims, const uint64_t *strides,
                  const uint32_t *box, Swizzle sw);
int make_tmap_typed(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, int rank, const uint64_t *dims,
                    const uint64_t *strides, const uint32_t *box, Swizzle sw);

}  // namespace tc
}  // namespace zb
