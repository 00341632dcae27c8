// Thin inline-PTX wrappers for sm_100a: mbarriers, 1-D bulk async copies
// (TMA engine, no tensor map), and bounded waits.
//
// No cluster multicast is used anywhere in this library.
#pragma once

#include <cstdint>
#include "axq_common.cuh"

namespace axq {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait that may suspend the thread for up to `ns` nanoseconds; the
// thread resumes as soon as the phase completes.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

// Global nanosecond timer.
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the phase with the given parity to complete.  Returns false if
// *abort_flag (shared memory, may be null) becomes set or kWaitLimitNs pass;
// the caller then reports an error status.  Waiting threads sleep in
// try_wait instead of polling, so they take no issue slots from the warps
// doing the work.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  const volatile int* abort_flag = nullptr) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, kSuspendNs)) return true;
        if (abort_flag && *abort_flag) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// dst, src and bytes must all be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// L2 policy for data read once (streamed weights): evicted first, so the
// small operands around it (activations, outputs) keep their L2 lines.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// bulk_g2s with an L2 cache policy.
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 16-byte asynchronous global -> shared copy (L2-cached, bypasses L1);
// both addresses 16-byte aligned.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Arrives on `bar` (counted as one of its expected arrivals) once every
// cp.async this thread issued before has completed.
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ int dp4a_s8(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// n little-endian 32-bit words starting at shared address p (any byte
// alignment).  Reads n+1 aligned words; the extra word may lie up to 4 bytes
// past the data, so shared buffers carry slack.
template <int N>
__device__ __forceinline__ void ld_words(const uint8_t* p, uint32_t* out) {
    // The aligned base is formed by pointer arithmetic (not an integer round
    // trip), so a pointer into shared memory stays one: the compiler then
    // emits shared loads instead of generic ones.
    const uint32_t mis = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p)) & 3u;
    const uint32_t* base = reinterpret_cast<const uint32_t*>(p - mis);
    const uint32_t sh = mis * 8;
    uint32_t w[N + 1];
#pragma unroll
    for (int i = 0; i <= N; ++i) w[i] = base[i];
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = __funnelshift_r(w[i], w[i + 1], sh);
}

// Programmatic dependent launch (sm_90+).  wait: block until the
// preceding kernel of the stream has completed and its writes are visible
// (returns at once when this grid was launched without the attribute).
// launch_dependents: allow the next kernel, if launched with the attribute,
// to be scheduled before this grid completes.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Acquire load at system scope (flags written by other GPUs).
__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Release fence at system scope: this thread's earlier writes (and those it
// has observed) are visible to every GPU before its later writes.
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Atomic add with acquire-release semantics at GPU scope; returns the old value.
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu_u32(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Relaxed atomic add at system scope without a return value (a signal
// counter on this or another GPU).
__device__ __forceinline__ void red_add_sys_u32(unsigned* p, unsigned v) {
    asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// CTA-scope release store / acquire load of a shared-memory word (a flag
// handed from one warp of the CTA to another).
__device__ __forceinline__ void st_release_cta_shared_u32(unsigned* p, unsigned v) {
    asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_cta_shared_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}

// Polls *p (acquire, system scope) until the counter has reached `target`
// ((int)(*p - target) >= 0, wrap-safe); false after limit_ns of global time.
// 8-byte relaxed store / load at system scope (slots read by other GPUs;
// single-copy atomic when 8-byte aligned).
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ bool poll_counter_sys(const unsigned* p, unsigned target, uint64_t limit_ns) {
    if (static_cast<int>(ld_acquire_sys_u32(p) - target) >= 0) return true;
    const uint64_t t0 = globaltimer_ns();
    while (static_cast<int>(ld_acquire_sys_u32(p) - target) < 0) {
        if (globaltimer_ns() - t0 > limit_ns) return false;
        __nanosleep(100);
    }
    return true;
}

__device__ __forceinline__ uint32_t byte_of(const uint32_t* w, int i) { return (w[i >> 2] >> (8 * (i & 3))) & 0xFFu; }

}  // namespace axq
