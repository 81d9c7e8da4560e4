// Thin inline-PTX wrappers for the sm_100a features the q6 kernels use:
// mbarriers (with bounded waits), TMA tile loads, TMEM allocation, tcgen05
// MMA / commit / ld / st and their ordering fences.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace q6 {

// Device-side error word, one per translation unit (the library is built
// without relocatable device code).  A bounded wait that gives up writes its
// site code here (first writer wins); each unit exposes a host accessor that
// q6_get_device_error() polls.
static __device__ int g_device_error = 0;

// A single mbarrier wait that takes longer than this is treated as a hang.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Rounds a dynamic shared-memory pointer up to kAlign bytes by pointer
// arithmetic on the shared array itself, so that the compiler keeps every
// pointer derived from it in the shared address space (a round trip through
// an integer makes each access through it a generic one).
template <uint32_t kAlign>
__device__ __forceinline__ uint8_t* smem_align_up(uint8_t* p) {
    return p + ((kAlign - (smem_u32(p) & (kAlign - 1u))) & (kAlign - 1u));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void record_error(int code) { atomicCAS(&g_device_error, 0, code); }

__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "selp.b32 %0, 1, 0, P;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread may sleep up to `hint_ns`
// inside the instruction and is woken when the phase completes, so waiting
// warps do not spin on issue slots the dequant warps need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2, %3;\n\t"
        "selp.b32 %0, 1, 0, P;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete.  Gives up (returns
// false) when the CTA-wide abort flag is raised or after limit_ns; in the
// latter case it raises the abort flag and records `site` in g_device_error.
// The clock is checked every 16 suspended tries (each sleeps at most `hint_ns`).
__device__ __forceinline__ bool mbar_wait_limit(uint32_t bar, uint32_t parity, volatile int* abort_flag, int site,
                                                uint64_t limit_ns, uint32_t hint_ns = 20000u) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_sleep(bar, parity, hint_ns)) return true;
        if ((i & 15u) == 0) {
            if (*abort_flag) return false;
            if (global_timer_ns() - t0 > limit_ns) {
                *abort_flag = 1;
                record_error(site);
                return false;
            }
        }
    }
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int site) {
    return mbar_wait_limit(bar, parity, abort_flag, site, kWaitLimitNs);
}

// Bounded wait that ignores the abort flag (used to drain in-flight copies
// before a CTA exits).
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
    return true;
}

// --------------------------------------------------------------------- TMA

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// 2-D tiled bulk tensor copy global -> this CTA's shared memory, completing
// `bytes` of transaction count on `bar`.  x is the innermost coordinate.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(map), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` of
// transaction count on `bar`.  Both addresses 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// ------------------------------------------------------------ CTA pairs
// A cluster of two CTAs sharing one cta_group::2 MMA: rank 0 (the leader)
// issues the MMAs for both; barriers the leader waits on collect arrivals
// from both CTAs.

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Shared::cluster address of this CTA's shared variable `addr` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

// Arrive on a barrier given by its shared::cluster address (this CTA's or the
// peer's), with the default (CTA-scope release) semantics: what it publishes
// is tensor-memory or accumulator state, ordered by the tcgen05 fences around
// it.  A cluster-scope release here costs 1-2 k cycles per arrival on B200.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 2-D tiled copy into this CTA's shared memory whose completion counts on a
// barrier of either CTA of the pair (`bar` a shared::cluster address).  No
// multicast: each CTA fetches its own half of the tile.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar, int32_t x,
                                                 int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(map), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// its later async-proxy ones (a bulk copy that overwrites a buffer just read).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------- TMEM

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

// Pair forms: both CTAs' allocating warps (same warp index) allocate the same
// columns; the leader's MMAs then address both CTAs' tensor memory.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive once on `bar` when every tcgen05 op this thread issued so far is done.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}

// Commit of the leader's pair MMAs, arriving on the barrier at the same
// shared-memory offset in every CTA of `mask` (bit r = cluster rank r).
__device__ __forceinline__ void tc_commit_pair(uint32_t bar, uint16_t mask) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::
                     "r"(bar), "h"(mask)
                 : "memory");
}

// Pair MMA issued by the leader: D rows 0-127 in the leader's tensor memory
// and 128-255 in the peer's, A likewise, B's N columns split in halves
// between the two CTAs' shared memory at the same offset.
__device__ __forceinline__ void mma_bf16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem)^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Instruction descriptor: bf16 A and B (both K-major), fp32 accumulator, MxN.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
    return (1u << 4)                              // D format: f32
           | (1u << 7)                            // A format: bf16
           | (1u << 10)                           // B format: bf16
           | (static_cast<uint32_t>(n >> 3) << 17)  // N / 8
           | (static_cast<uint32_t>(m >> 4) << 24); // M / 16
}

__device__ __forceinline__ uint64_t make_desc(uint32_t lo, uint32_t hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
    return d;
}

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzling: rows of 64 bf16 (128 B), 8-row swizzle atoms 1024 B
// apart.  The tile base must be 1024-byte aligned; stepping K by 16 elements
// inside the atom adds 32 B to the start address.
__device__ __forceinline__ uint64_t sdesc_kmajor_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);  // start address
    d |= static_cast<uint64_t>(1u) << 16;                      // leading byte offset (unused)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;              // stride byte offset
    d |= static_cast<uint64_t>(1u) << 46;                      // sm_100 descriptor version
    d |= static_cast<uint64_t>(2u) << 61;                      // 128-byte swizzle
    return d;
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp writes lane
// (lane field of taddr) + i.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
        "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
        "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
          "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
          "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
          "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
          "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// --------------------------------------------------------------- programmatic dependent launch
// A kernel launched with programmatic stream serialization may start while
// the previous kernel of the stream is still running (once every CTA of that
// kernel has executed pdl_launch_dependents, or it has completed).  Before
// its first read of anything the previous kernel may have written, and its
// first global write, it must execute pdl_wait: that returns once the
// previous grids have completed and their memory is visible.  Weights are
// never written by these kernels, so their prefetch may precede the wait.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// --------------------------------------------------------------- numerics

__device__ __forceinline__ float tanh_fast(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// GELU with the tanh approximation, 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))),
// the formula of mlx nn.gelu_approx used by the reference epilogue.  The fast
// form takes the hardware tanh.approx.f32 (about 2^-11 relative error); the
// precise form CUDA's tanhf, for callers that ask for the reference kernel's
// metal::precise::tanh (Q6_EPI_GELU_PRECISE).
__device__ __forceinline__ float gelu_tanh(float x) {
    const float x3 = x * x * x;
    const float inner = 0.7978845608028654f * (x + 0.044715f * x3);
    return 0.5f * x * (1.0f + tanh_fast(inner));
}

__device__ __forceinline__ float gelu_tanh_precise(float x) {
    const float x3 = x * x * x;
    const float inner = 0.7978845608028654f * (x + 0.044715f * x3);
    return 0.5f * x * (1.0f + tanhf(inner));
}

__device__ __forceinline__ float gelu_select(float x, bool precise) {
    return precise ? gelu_tanh_precise(x) : gelu_tanh(x);
}

// The same GELU on two values with packed fp32x2 arithmetic:
// 0.5x + 0.5x * tanh(x (k + k c x^2)), k = sqrt(2/pi), c = 0.044715.
__device__ __forceinline__ float2 gelu_tanh2(float2 x) {
    constexpr float k = 0.7978845608028654f;
    constexpr float kc = 0.7978845608028654f * 0.044715f;
    const float2 x2 = __fmul2_rn(x, x);
    const float2 inner = __fmul2_rn(x, __ffma2_rn(make_float2(kc, kc), x2, make_float2(k, k)));
    const float2 t = make_float2(tanh_fast(inner.x), tanh_fast(inner.y));
    const float2 h = __fmul2_rn(make_float2(0.5f, 0.5f), x);
    return __ffma2_rn(h, t, h);
}

__device__ __forceinline__ float2 gelu_tanh2_select(float2 x, bool precise) {
    if (precise) return make_float2(gelu_tanh_precise(x.x), gelu_tanh_precise(x.y));
    return gelu_tanh2(x);
}

}  // namespace q6
