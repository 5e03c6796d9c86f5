// rkb_ptx.cuh -- thin inline-PTX wrappers for the sm_100a primitives the
// kernels of this library use: mbarriers with bounded waits, TMA tensor and
// bulk loads, tcgen05 TMEM allocation / MMA / commit / loads, and the shared
// memory matrix descriptors the MMA reads operands through.
//
// Every wait on an mbarrier is bounded: after RKB_WAIT_NS of wall time (read
// from %globaltimer) the waiter records an error code in the caller-supplied
// error word and gives up, and every other waiter that sees the word set also
// gives up, so a kernel whose pipeline stalls returns with a status instead of
// hanging the GPU.
#pragma once
#include <stdint.h>
#include <cuda.h>
#include <cuda_runtime.h>

#define RKB_DEV __device__ __forceinline__

#ifndef RKB_WAIT_NS
#define RKB_WAIT_NS 2000000000ull   // 2 s: legitimate waits here last microseconds
#endif

namespace rkb {

// Error codes written to the device error word (first writer wins).
enum : int {
    ERR_NONE = 0,
    ERR_WAIT_PRODUCER = 1,   // TMA producer waited too long for a free stage
    ERR_WAIT_MMA_FULL = 2,   // MMA issuer waited too long for a loaded stage
    ERR_WAIT_MMA_ACC  = 3,   // MMA issuer waited too long for a drained accumulator
    ERR_WAIT_EPILOGUE = 4,   // epilogue waited too long for a finished accumulator
    ERR_WAIT_DEQUANT  = 5,   // dequant warps waited too long for raw weights / a free slot
    ERR_WAIT_DRAIN    = 6,   // final drain of in-flight MMAs timed out
};

RKB_DEV uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

RKB_DEV uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Hardware base-2 exponential (MUFU, flush-to-zero).  Used for softmax
// weights.  With lazy rescaling (the running max is only moved when a row max
// grows by more than 2^8 in log2 units) the arguments are <= 8, so weights are
// < 2^8 (safe in fp16) and -inf gives 0; row sums and O stay in fp32.  The
// ~2 ulp error is far below fp16 resolution.
RKB_DEV float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// One lane of a converged warp (the lowest active one); the same on every
// lane of the warp.  Lets a whole warp run an MMA-issuing loop (so the
// loop's addresses and descriptors stay warp-uniform) while exactly one
// thread issues each tcgen05 instruction.
RKB_DEV bool elect_one() {
    uint32_t pred;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "elect.sync _|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(pred));
    return pred != 0;
}

// ---- mbarriers -------------------------------------------------------------
RKB_DEV void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
RKB_DEV void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
RKB_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// Non-blocking test: never suspends the thread.
RKB_DEV bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}

// Non-blocking tries before the blocking wait.  0 by default: spinning warps
// take issue slots from the warps doing work, which cost the GEMMs 3-5 %.  The
// attention kernel, whose roles hand off every 128-key block, sets 4096 (its
// block rate rose ~20 %).
#ifndef RKB_SPIN_TRIES
#define RKB_SPIN_TRIES 0
#endif

// Bounded wait for the phase of parity `parity` to complete.  Returns false if
// the wait expired (error recorded) or another role already recorded an error.
// The first RKB_SPIN_TRIES tries use the non-blocking test, so a phase that
// completes within several microseconds is seen at once (a blocking try_wait
// that finds the phase incomplete may suspend the thread for a hardware-chosen
// time); then try_wait, which takes no issue slots while suspended.
RKB_DEV bool mbar_wait(uint32_t bar, uint32_t parity, int *err, int code) {
    for (int i = 0; i < RKB_SPIN_TRIES; ++i)
        if (mbar_test_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        // The error word may live in mapped host memory: poll it (and the
        // clock) only every 1024 tries so spinning warps do not flood PCIe.
        if ((i & 1023u) == 0) {
            if (*reinterpret_cast<volatile int *>(err) != 0) return false;
            if (global_timer_ns() - t0 > RKB_WAIT_NS) {
                // plain store: the word may be mapped host memory, where device
                // atomics are not atomic anyway; any non-zero code is an error
                *reinterpret_cast<volatile int *>(err) = code;
                return false;
            }
        }
    }
}
// Warp-wide wait with one polling lane: lane 0 waits (acquire), then the warp
// converges at __syncwarp, which orders lane 0's observation before every
// lane's later accesses.  Keeps 31 lanes off the barrier's shared-memory word.
// Returns the same value in every lane.
RKB_DEV bool mbar_wait_warp(uint32_t bar, uint32_t parity, int *err, int code) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, err, code) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}
// Bounded wait that ignores the error word (used to drain in-flight async work
// on an error path).  Returns false on expiry.
RKB_DEV bool mbar_wait_drain(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_timer_ns() - t0 > RKB_WAIT_NS) return false;
    return true;
}
RKB_DEV void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
RKB_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

// ---- TMA ---------------------------------------------------------------------
// 2D tiled tensor load, no multicast.  c0 is the inner (contiguous) coordinate
// in elements; callers keep c0 * element size a multiple of 16 bytes.
RKB_DEV void tma_load_2d(uint32_t dst, const CUtensorMap *tm, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}
// Pull a 2D tile into L2 ahead of its shared-memory load (no completion
// tracking, no shared memory used).
RKB_DEV void tma_prefetch_2d(const CUtensorMap *tm, int c0, int c1) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];"
                 ::"l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1) : "memory");
}
// Contiguous bulk copy global -> shared (no tensor map).  dst, src 16-byte
// aligned and bytes a multiple of 16.
RKB_DEV void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
        : "memory");
}
RKB_DEV void prefetch_tmap(const CUtensorMap *tm) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}
// Make generic-proxy writes to shared memory visible to the async proxy (the
// tensor core reads operands through it).
RKB_DEV void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 2D tiled TMA store shared -> global (out-of-range rows / columns are not
// written), tracked by bulk async-groups of the issuing thread.
RKB_DEV void tma_store_2d(const CUtensorMap *tm, uint32_t src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(tm)), "r"(src), "r"(c0), "r"(c1) : "memory");
}
RKB_DEV void tma_store_3d(const CUtensorMap *tm, uint32_t src, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(tm)), "r"(src), "r"(c0), "r"(c1), "r"(c2) : "memory");
}
RKB_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most N of this thread's bulk groups still read shared memory
template <int N> RKB_DEV void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// wait until at most N of this thread's bulk groups are incomplete
template <int N> RKB_DEV void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ---- tcgen05 -------------------------------------------------------------------
RKB_DEV void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(dst_smem), "r"(ncols) : "memory");
}
RKB_DEV void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
RKB_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
RKB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
RKB_DEV void tc_fence_after()  { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on `bar` once every tcgen05.mma issued so far by this thread completes.
RKB_DEV void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(bar) : "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, fp16/bf16 inputs.
RKB_DEV void tc_mma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accum) : "memory");
}
// D(tmem) (+)= A * B^T, tf32 inputs (fp32 storage), fp32 accumulate.
RKB_DEV void tc_mma_tf32(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accum) : "memory");
}
// D(tmem) (+)= A * B^T, signed/unsigned 8-bit inputs, int32 accumulate.
RKB_DEV void tc_mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accum) : "memory");
}

// Warp-collective load of 32 consecutive 32-bit TMEM columns for the warp's 32
// lanes (thread i gets lane base+i).
RKB_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}
RKB_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- CTA pairs (cta_group::2) ---------------------------------------------------
// A cluster of two CTAs on two SMs shares one MMA: the leader (rank 0) issues
// tcgen05.mma.cta_group::2 reading A and B halves from both CTAs' shared
// memory and writing both CTAs' TMEM.  No multicast is used anywhere: each CTA
// loads its own halves, and peer barriers are signalled through mapa addresses.
RKB_DEV uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
RKB_DEV void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same shared::cta offset in CTA `rank`.
RKB_DEV uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
RKB_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 2D tiled load whose completion is counted on the leader CTA's barrier
// (`bar` is a shared::cluster address of that barrier).  No multicast.
RKB_DEV void tma_load_2d_pair(uint32_t dst, const CUtensorMap *tm, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}
RKB_DEV void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(dst_smem), "r"(ncols) : "memory");
}
RKB_DEV void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
RKB_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
// Arrive on the barrier at shared::cluster address `bar` (own or peer CTA) once
// every cta_group::2 MMA issued so far by this thread completes.
RKB_DEV void tc_commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(bar) : "memory");
}
RKB_DEV void tc_mma_f16_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accum) : "memory");
}
RKB_DEV void tc_mma_tf32_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accum) : "memory");
}
RKB_DEV void tc_mma_i8_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accum) : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle (rows of 128 bytes, 8-row / 1024-byte swizzle atoms, which is
// what a TMA load with CU_TENSOR_MAP_SWIZZLE_128B writes):
//   bits  0-13 start address >> 4        bits 16-29 leading byte offset >> 4 (unused: 1)
//   bits 32-45 stride byte offset >> 4 (1024 B between 8-row groups)
//   bits 46-47 descriptor version (1 on sm_100)   bits 61-63 layout (2 = SWIZZLE_128B)
// The tile base must be 1024-byte aligned; stepping K inside the 128-byte row is
// done by advancing the start address.
RKB_DEV uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(1) << 16;
    d |= static_cast<uint64_t>(1024 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// Instruction descriptors (kind::f16 and kind::i8), both operands K-major, dense.
//   bits 4-5 accumulator format (1 = f32, 2 = s32), bits 7-9 / 10-12 A / B format
//   (f16: 0 = f16, 1 = bf16; i8: 1 = signed), bits 17-22 N >> 3, bits 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16_f32acc(int m, int n) {
    return (1u << 4) | (0u << 7) | (0u << 10) |
           (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}
// kind::f16 with bf16 operands (format 1) / kind::tf32 (format 2), fp32 accumulate
__host__ __device__ constexpr uint32_t idesc_f32acc_fmt(int fmt, int m, int n) {
    return (1u << 4) | (static_cast<uint32_t>(fmt) << 7) | (static_cast<uint32_t>(fmt) << 10) |
           (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_s8_s32acc(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) |
           (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

}  // namespace rkb
