// sm_100a building blocks: mbarriers, tcgen05 (TMEM alloc, MMA, commit, ld),
// shared-memory matrix descriptors, bulk async copies and bounded waits.
//
// Every wait in this engine is bounded: a wait that runs past its limit sets a
// device-side error word (read back by the host after the frame) and returns
// false, so a bad descriptor or a lost arrive ends the kernel instead of
// hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace dnb {

// Device error word layout (one uint32 per engine instance):
//   0 = ok, otherwise (site << 16) | code.
enum : uint32_t {
    kErrMbarTimeout = 1,
    kErrTmemAlloc = 2,
    kErrBadShape = 3,
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void report_error(uint32_t* err, uint32_t site, uint32_t code) {
    if (err) atomicCAS(err, 0u, (site << 16) | code);
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bring a kernel-parameter tensor map into the TMA descriptor cache, so that
// the first copy after the grid-dependency wait does not fetch it.
__device__ __forceinline__ void prefetch_tmap(const void* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Bounded wait on an mbarrier phase. Gives up after `limit_ns` of wall time
// (checked every 64 polls) and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0u && globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// Bounded wait shared by the roles of a warp-specialised kernel: gives up
// as soon as another role has set `abort_flag`, and on its own timeout
// records `site` in the error word and sets the flag for the others.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                              uint32_t* err, uint32_t site) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0u) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > 2000000000ull) {
                report_error(err, site, kErrMbarTimeout);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// Named barrier `id` over `n` threads (a multiple of 32).
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Same barrier, returning the OR of `v` over its threads (a decision that is
// uniform across them).
__device__ __forceinline__ bool named_sync_or(uint32_t id, uint32_t n, bool v) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(out)
        : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(n)
        : "memory");
    return out != 0;
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// 1-D bulk copy global -> shared through the TMA engine, completion counted
// on `bar` in bytes. src/dst 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---------------------------------------------------------------------------
// cp.async (16-byte, L2-only) for gathers that a bulk copy cannot express
// ---------------------------------------------------------------------------

__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src_gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)),
                 "l"(src_gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async16_zfill(void* dst_smem, const void* src_gmem, bool valid) {
    const uint32_t n = valid ? 16u : 0u;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst_smem)),
                 "l"(src_gmem), "r"(n)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------
// Fences
// ---------------------------------------------------------------------------

// Make generic-proxy shared-memory writes visible to the async proxy (the
// tensor core reads operands through it).
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMEM allocation (one warp executes these)
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
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

// ---------------------------------------------------------------------------
// UMMA descriptors
// ---------------------------------------------------------------------------

// Shared-memory matrix descriptor, K-major, no swizzle ("interleaved"):
// the operand is stored as core matrices of 8 rows x 16 bytes (128 contiguous
// bytes, row stride 16 B). `lbo` = byte distance between core matrices that
// are adjacent along K, `sbo` = byte distance between adjacent 8-row groups.
__device__ __forceinline__ uint64_t sdesc_kmajor(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
    return d;                             // base offset 0, layout type 0 (no swizzle)
}

// Shared-memory matrix descriptor, K-major, swizzled (the layout a TMA load
// with CU_TENSOR_MAP_SWIZZLE_{32,64,128}B writes): rows of `row_bytes`
// (32/64/128) with 16-byte chunks XOR-permuted within each 8-row atom.
// SBO = 8 rows; LBO is unused for K-major swizzled operands. Advance the
// start address by 32 bytes per K=16 step inside the row.
__device__ __forceinline__ uint64_t sdesc_kmajor_sw(uint32_t saddr, uint32_t row_bytes) {
    const uint32_t layout = row_bytes == 128 ? 2u : (row_bytes == 64 ? 4u : 6u);
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;                           // LBO (unused)
    d |= static_cast<uint64_t>(((8u * row_bytes) >> 4) & 0x3FFFu) << 32;  // SBO
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(layout) << 61;
    return d;
}

// The same descriptor with its start address moved by `bytes` (a multiple of
// 16). An MMA issue loop builds its descriptors once and steps them with this
// add: rebuilding them per MMA from runtime values puts ~100+ cycles of
// integer work before every tcgen05.mma of the single issuing thread, which
// then issues well below the tensor core's rate.
__device__ __forceinline__ uint64_t desc_add(uint64_t desc, uint32_t bytes) { return desc + (bytes >> 4); }

// Byte offset of 16-byte chunk j of row r in a swizzled K-major tile whose
// rows are `row_bytes` long (the TMA swizzle pattern of that span).
__device__ __forceinline__ uint32_t sw_offset(uint32_t r, uint32_t j, uint32_t row_bytes) {
    const uint32_t sw = row_bytes == 128 ? (r & 7u) : (row_bytes == 64 ? ((r >> 1) & 3u) : ((r >> 2) & 1u));
    return r * row_bytes + ((j ^ sw) << 4);
}

// Instruction descriptor for tcgen05.mma kind::f16 with fp16 A/B, fp32
// accumulate, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
    return (1u << 4)                                   // D format: f32
           | (0u << 7) | (0u << 10)                    // A, B: f16
           | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
           | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

// Byte offset of element (row, k) in the no-swizzle K-major layout with
// core matrices contiguous along K (lbo = 128) and `kbytes_row` = K*2 bytes
// per 8-row group stride factor: sbo = (K/8)*128.
__host__ __device__ __forceinline__ uint32_t kmajor_offset(uint32_t row, uint32_t kchunk,
                                                           uint32_t sbo) {
    return (row >> 3) * sbo + kchunk * 128u + (row & 7u) * 16u;
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by a single thread.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once all previously issued MMAs of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// ---------------------------------------------------------------------------
// TMEM -> registers (32 lanes x 32 bit, 16 or 32 columns per call)
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// TMEM address of (lane, column).
__device__ __forceinline__ uint32_t tmem_addr(uint32_t base, uint32_t lane, uint32_t col) {
    return base + (lane << 16) + col;
}

// ---------------------------------------------------------------------------
// Small numeric helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_half2(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
}

// ---------------------------------------------------------------------------
// fp16 vectors, TMA tensor copies, bulk groups
// ---------------------------------------------------------------------------

__device__ __forceinline__ void h8_to_f(const uint4& v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = unpack_half2(w[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

__device__ __forceinline__ uint4 f_to_h8(const float (&f)[8]) {
    uint4 v;
    v.x = pack_half2(f[0], f[1]);
    v.y = pack_half2(f[2], f[3]);
    v.z = pack_half2(f[4], f[5]);
    v.w = pack_half2(f[6], f[7]);
    return v;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const void* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const void* map, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const void* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_store_2d(const void* map, int c0, int c1, const void* src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(smem_u32(src))
                 : "memory");
}

__device__ __forceinline__ void tma_store_3d(const void* map, int c0, int c1, int c2, const void* src) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src))
                 : "memory");
}

__device__ __forceinline__ void tma_store_4d(const void* map, int c0, int c1, int c2, int c3, const void* src) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(src))
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read1() {
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Packed fp32 FMA (two lanes per instruction on sm_100): d = a * b + c.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long ra, rb, rc, rd;
    memcpy(&ra, &a, 8);
    memcpy(&rb, &b, 8);
    memcpy(&rc, &c, 8);
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
    float2 d;
    memcpy(&d, &rd, 8);
    return d;
}

// Mixed-precision FMA on the two halves of packed fp16 pairs (sm_100):
// c0 += lo(u) * lo(w), c1 += hi(u) * hi(w) in fp32. A product of two fp16
// values is exact in fp32, so this equals fmaf on the widened operands
// without the two conversions.
__device__ __forceinline__ void fma_mix2(float& c0, float& c1, uint32_t u, uint32_t w) {
    asm("{\n\t.reg .f16 ul, uh, wl, wh;\n\t"
        "mov.b32 {ul, uh}, %2;\n\t"
        "mov.b32 {wl, wh}, %3;\n\t"
        "fma.rn.f32.f16 %0, ul, wl, %0;\n\t"
        "fma.rn.f32.f16 %1, uh, wh, %1;\n\t}"
        : "+f"(c0), "+f"(c1)
        : "r"(u), "r"(w));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (a cluster of two CTAs sharing tcgen05 MMAs: cta_group::2)
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// The shared::cluster address of `bar` (a variable of this CTA's shared
// memory) in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(const void* bar, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(bar)), "r"(rank));
    return a;
}

// Arrive (release at cluster scope) on an mbarrier of another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// Every thread of both CTAs of the cluster: the barrier initialisation of
// each CTA is visible to the other before either arrives remotely.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMEM of a CTA pair: one warp of each CTA (the same warp index) allocates,
// relinquishes and frees; each CTA's TMEM gets the same columns.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem of both CTAs] (+)= A[128 rows of each CTA's smem] * B[N/2 rows of each
// CTA's smem]^T: one M = 256 MMA of the pair, issued by one thread of the
// even CTA; the descriptors' addresses hold in both CTAs.
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` (same offset) in both CTAs of the pair once all previously
// issued pair MMAs of this thread complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(static_cast<uint16_t>(3))
        : "memory");
}

}  // namespace dnb
