// common.cuh — shared device/host helpers for the sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>
#include <utility>

#include "../../include/aaedn_b200.h"
#include "../host/host_common.hpp"

namespace aaedn_dev
{

using aaedn_host::set_error;

// Kernels launched by this library (host-side count, graph replays add the
// per-step node count).
extern std::atomic<uint64_t> g_launches;
inline void count_launch(uint64_t n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

#define AAEDN_CUDA_TRY(expr)                                                                                  \
    do                                                                                                        \
    {                                                                                                         \
        cudaError_t _e = (expr);                                                                              \
        if (_e != cudaSuccess)                                                                                \
            return ::aaedn_host::set_error(AAEDN_ECUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), \
                                           __FILE__, __LINE__);                                               \
    } while (0)

#define AAEDN_LAUNCH_CHECK(name)                                                                              \
    do                                                                                                        \
    {                                                                                                         \
        cudaError_t _e = cudaGetLastError();                                                                  \
        if (_e != cudaSuccess)                                                                                \
            return ::aaedn_host::set_error(AAEDN_ECUDA, "launch of %s failed: %s", name, cudaGetErrorString(_e)); \
        ::aaedn_dev::count_launch();                                                                          \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// SMs of the current device (cached per device).
inline int sm_count()
{
    static int cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64)
        dev = 0;
    if (!cache[dev])
    {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

// A set-up step that must run once on every device a process uses, such as
// cudaFuncSetAttribute (it acts on the current device only). Thread-safe:
// the first caller on a device runs it under the lock; later callers, and
// callers on devices where it already succeeded, return at once.
class PerDeviceOnce
{
  public:
    template <typename Fn>
    int run(Fn&& fn)
    {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess)
            return set_error(AAEDN_ECUDA, "cudaGetDevice failed: %s", cudaGetErrorString(e));
        if (dev < 0 || dev >= 64)
            return set_error(AAEDN_EUNSUPPORTED, "device ordinal %d >= 64", dev);
        const uint64_t bit = 1ull << dev;
        if (done_.load(std::memory_order_acquire) & bit)
            return AAEDN_OK;
        std::lock_guard<std::mutex> lk(mu_);
        if (done_.load(std::memory_order_relaxed) & bit)
            return AAEDN_OK;
        const int rc = fn();
        if (rc == AAEDN_OK)
            done_.fetch_or(bit, std::memory_order_release);
        return rc;
    }

  private:
    std::mutex mu_;
    std::atomic<uint64_t> done_{0};
};

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Scale decode: 0 = IEEE fp16 bits, 1 = integer cast (src/dequant.cpp:19).
template <int SK>
__device__ __forceinline__ float decode_scale(uint16_t s)
{
    if constexpr (SK == AAEDN_SCALE_F16)
        return __half2float(__ushort_as_half(s));
    else
        return (float)s;
}

// Streaming 16-byte load of weights: read once, do not keep in L1.
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint16_t ldg_u16(const uint16_t* p)
{
    uint16_t r;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ float4 ldg_stream_f4(const float* p)
{
    float4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p));
    return r;
}

// two bf16 (lo = first element) in one 32-bit register
__device__ __forceinline__ uint32_t pack_bf16(__nv_bfloat16 lo, __nv_bfloat16 hi)
{
    return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}

// D += A(16x16 bf16, row) * B(16x8 bf16, col), fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float& d0, float& d1, float& d2, float& d3, uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d0), "+f"(d1), "+f"(d2), "+f"(d3)
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Nibble pairs of one 32-bit weight word (8 codes, code i in bits 4i..4i+3)
// as bf16x2 values 16 + code: the code lands in mantissa bits 3..6 of each
// half under the exponent of 16.0 (0x4180). E0 = codes (0,4), E1 = (1,5),
// E2 = (2,6), E3 = (3,7).
// (x & 0x00780078) | 0x41804180 as one LOP3 (truth table 0xEA = (a & b) | c)
__device__ __forceinline__ uint32_t lop3_bias(uint32_t x)
{
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(x), "n"(0x00780078), "n"(0x41804180));
    return d;
}
__device__ __forceinline__ uint32_t nib_e0(uint32_t w) { return lop3_bias(w << 3); }
__device__ __forceinline__ uint32_t nib_e1(uint32_t w) { return lop3_bias(w >> 1); }
__device__ __forceinline__ uint32_t nib_e2(uint32_t w) { return lop3_bias(w >> 5); }
__device__ __forceinline__ uint32_t nib_e3(uint32_t w) { return lop3_bias(w >> 9); }
// (16 + c) - 16 = c on both halves of a bf16x2 word: exact (4-bit integers
// are exact in bf16), so the codes enter the product without a bias to
// remove after the accumulation.
__device__ __forceinline__ uint32_t unbias16(uint32_t v)
{
    uint32_t r;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(0x41804180u));
    return r;
}

// D += A (16x32 u8, row) * B (32x8 s8, col) with s32 accumulators: the dot
// product engine of the integer GEMV (exact: no rounding anywhere).
__device__ __forceinline__ void mma_u8s8_16832(int& d0, int& d1, int& d2, int& d3, uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+r"(d0), "+r"(d1), "+r"(d2), "+r"(d3)
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

// ---- asynchronous global -> shared copies (per-thread, L2 only) ----------
__device__ __forceinline__ uint32_t smem_addr(const void* p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

// 16 bytes; src_bytes == 0 writes zeros without reading global memory.
__device__ __forceinline__ void cp_async_16(void* dst, const void* src, uint32_t src_bytes)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}

// 16 bytes of a stream that continues at the following addresses: L2 fetches
// the surrounding 256 bytes from DRAM in one request.
__device__ __forceinline__ void cp_async_16_pf256(void* dst, const void* src, uint32_t src_bytes)
{
    asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}

// 4 bytes (cache at all levels form: .ca is the only one allowed below 16 B)
__device__ __forceinline__ void cp_async_4(void* dst, const void* src, uint32_t src_bytes)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr)
{
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
    return r;
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr)
{
    uint32_t r;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r) : "r"(addr));
    return r;
}

__device__ __forceinline__ float ldsf(uint32_t addr)
{
    float r;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(r) : "r"(addr));
    return r;
}

__device__ __forceinline__ float2 lds64f(uint32_t addr)
{
    float2 r;
    asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(r.x), "=f"(r.y) : "r"(addr));
    return r;
}

// Packed fp32 pairs (sm_100): each component rounds exactly as mul.rn /
// fma.rn of one float, so these are __fmul_rn / fmaf on two lanes of data
// in one instruction.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b)
{
    float2 d;
    asm("{\n\t.reg .b64 pa, pb, pd;\n\t"
        "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
        "mul.rn.f32x2 pd, pa, pb;\n\tmov.b64 {%0, %1}, pd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// a * b + c per component, one rounding (fmaf on each lane of the pair)
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c)
{
    float2 d;
    asm("{\n\t.reg .b64 pa, pb, pc, pd;\n\t"
        "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\tmov.b64 pc, {%6, %7};\n\t"
        "fma.rn.f32x2 pd, pa, pb, pc;\n\tmov.b64 {%0, %1}, pd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// ---- mbarriers and bulk (TMA) copies --------------------------------------
__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t addr, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(addr), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// arrive (count 1) and announce tx bytes that bulk copies will complete
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t addr, uint32_t tx)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(addr), "r"(tx) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t addr)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(addr), "r"(parity)
                 : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete, for at most
// limit_ns; false when the limit ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t addr, uint32_t parity, uint64_t limit_ns)
{
    if (mbar_try_wait(addr, parity))
        return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(addr, parity))
        if (globaltimer_ns() - t0 > limit_ns)
            return false;
    return true;
}

// global -> shared bulk copy completing on an mbarrier (size multiple of 16,
// both addresses 16-byte aligned)
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(mbar)
                 : "memory");
}

// L2 policy for data read once per step (the weight stream): evicted first,
// so it does not push the small hot data (activations, norms, recent KV
// rows) out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy()
{
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Timeline of one traced decode step: up to STEP_TRACE_CTAS CTAs of a launch
// each write STEP_TRACE_EVENTS globaltimer stamps (0 entry, 1 operand ready,
// 2 first weights arrived, 3 exit; 0 where a kernel has no such event).
constexpr int STEP_TRACE_CTAS = 1024;
constexpr int STEP_TRACE_EVENTS = 4;
__device__ __forceinline__ void trace_mark(unsigned long long* t, int cta, int e)
{
    if (t && cta < STEP_TRACE_CTAS)
        t[(size_t)cta * STEP_TRACE_EVENTS + e] = globaltimer_ns();
}

// Per-chunk stamps of a tiled GEMV's first STEP_TRACE_CHUNK_CTAS CTAs (consumer
// warp 0: chunk arrived, chunk released), after the per-CTA slots of its grid:
// slot (STEP_TRACE_CHUNK_BASE + cta * 2 * STEP_TRACE_CHUNKS + 2 q + e).
constexpr int STEP_TRACE_CHUNK_CTAS = 8, STEP_TRACE_CHUNKS = 24;
constexpr int STEP_TRACE_CHUNK_BASE = 160 * STEP_TRACE_EVENTS;
__device__ __forceinline__ void trace_chunk(unsigned long long* t, int cta, uint32_t q, int e)
{
    if (t && cta < STEP_TRACE_CHUNK_CTAS && q < (uint32_t)STEP_TRACE_CHUNKS)
        t[STEP_TRACE_CHUNK_BASE + (size_t)cta * 2 * STEP_TRACE_CHUNKS + 2 * q + e] = globaltimer_ns();
}

// Thread-block cluster barrier (every thread of every CTA of the cluster,
// convergent): the CTAs' shared-memory writes before it are visible to the
// cluster's reads after it.
__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// A float in the shared memory of CTA `rank` of this cluster, at the offset of
// the local shared address `laddr`.
__device__ __forceinline__ float ld_dsmem_f32(uint32_t laddr, uint32_t rank)
{
    uint32_t ra;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(laddr), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
    return v;
}

// bulk_g2s with an L2 cache policy
__device__ __forceinline__ void bulk_g2s_hint(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar,
                                              uint64_t policy)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, "
                 "[%3], %4;" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(mbar), "l"(policy)
                 : "memory");
}

// named barrier over `count` threads (warps 0..count/32-1)
__device__ __forceinline__ void named_bar_sync(int id, int count)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// named barrier that also ORs a predicate over the `count` threads: every
// thread gets the same answer (failure decisions taken together, so no thread
// leaves a loop whose barrier the others still wait at)
__device__ __forceinline__ bool named_bar_or(int id, int count, bool pred)
{
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\t"
                 "selp.u32 %0, 1, 0, q;\n\t}"
                 : "=r"(r)
                 : "r"((uint32_t)pred), "r"(id), "r"(count)
                 : "memory");
    return r != 0;
}

// ---- programmatic dependent launch ----------------------------------------
// Lets the next kernel in the stream start launching (its blocks then run
// their independent prologue: weight prefetch) ...
__device__ __forceinline__ void pdl_launch_dependents()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// ... and blocks until the previous kernel has completed and its writes are
// visible. A no-op when the kernel was not launched as a dependent.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Kernel launch, optionally as a programmatic dependent of the previous
// kernel in the stream (it may start while that one drains; it must call
// pdl_wait() before touching that kernel's outputs).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 bool pdl, Args&&... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

} // namespace aaedn_dev
