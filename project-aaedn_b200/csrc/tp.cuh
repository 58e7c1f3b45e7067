// tp.cuh — tensor parallelism of the decode step over T GPUs of one node.
//
// Rank r of T holds heads [r H/T, (r+1) H/T) (column-parallel qkv, its share
// of the KV cache), rows [r F/T, (r+1) F/T) of gate and up, the matching
// input columns of o and down (row-parallel), and lm_head rows [r V/T, ...).
// After o and down each rank has a partial sum of the full hidden-size
// output; instead of a library all-reduce, the GEMV's epilogue stores its rows
// in this rank's slot of its own receive buffer, and the GEMV's last CTA copies
// the whole slot into every other rank's receive buffer (CUDA IPC over
// NVLink) and raises a flag in each rank's memory. tp_reduce_kernel then
// waits for all flags and adds the T partials (read from its own memory, in
// rank order: the same sum, bit for bit, on every rank) to the residual.
// The greedy argmax is exchanged the same way, so all ranks feed
// the same token to the next step.
//
// Flags carry an epoch, E = tp_epoch + phase + 1, that only grows (phase:
// 2 per layer, then the argmax); tp_epoch advances by one step's worth in a
// one-thread kernel at the end of every captured step, so a wait never
// confuses steps. Partials are double
// buffered (o and down), so a rank can not overwrite a partial a peer has
// not read yet: it writes the o partial of layer l + 1 only after its down
// reduction of layer l saw every peer's down flag, which each peer raised
// after finishing its o reduction of layer l. Every wait is bounded
// (TP_WAIT_LIMIT_NS); a timed-out wait sets DecodeState::err = 4 and the
// kernel goes on without the missing data (the host reports the error).
#pragma once

#include "gemv_q4.cuh"

namespace aaedn_dev
{

struct TpReduceParams
{
    TpComm c;
    float* hidden;       // residual stream (local)
    int dim;
    int buf;             // 0: o partials, 1: down partials
    int phase;           // epoch offset of this reduction within the step
    int signal;          // also raise this rank's flag (0: the GEMV did)
    const unsigned* epoch;
    DecodeState* state;
};

// hidden[i] += sum over ranks (in rank order) of part[rank][buf][i]. Launched
// right after the GEMV that wrote this rank's partial (as its programmatic
// dependent: the launch wait returns once that kernel has finished). Block 0
// signals; every block waits for all flags.
__global__ void __launch_bounds__(256) tp_reduce_kernel(const TpReduceParams p)
{
    __shared__ int s_ok;
    // launched as a programmatic dependent of the GEMV that wrote this rank's
    // partial: everything below waits for that kernel
    pdl_launch_dependents();
    pdl_wait();
    const unsigned E = *p.epoch + (unsigned)p.phase + 1u;
    if (threadIdx.x == 0)
    {
        if (blockIdx.x == 0 && p.signal)
            tp_signal(p.c, E);
        s_ok = tp_wait_flags(p.c, E, p.state) ? 1 : 0;
    }
    __syncthreads();
    if (!s_ok)
        return;
    const float* rb = p.c.recv[p.c.rank] + (size_t)p.buf * p.dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.dim; i += gridDim.x * blockDim.x)
    {
        float s = 0.0f;
        for (int w = 0; w < p.c.size; ++w) // fixed order: the same sum on every rank
            s += __ldcg(rb + (size_t)w * 2 * p.dim + i);
        p.hidden[i] = __ldcg(p.hidden + i) + s; // residual (src/transformer.cpp:214)
    }
}

struct TpArgmaxParams
{
    TpComm c;
    const float* part_val; // this rank's per-CTA lm_head results (global token ids)
    const int* part_idx;
    int n_parts;
    int phase;
    const unsigned* epoch;
    DecodeState* state;
    uint32_t* out_tokens;
    int max_seq;
};

__device__ __forceinline__ void better(float& v, int& i, float ov, int oi)
{
    if (ov > v || (ov == v && oi < i))
    {
        v = ov;
        i = oi;
    }
}

// One block: this rank's best over its lm_head CTAs, exchanged with the
// peers; every rank then applies the same global argmax (ties to the lowest
// id) to its decode state and advances the epoch.
__global__ void __launch_bounds__(256) tp_argmax_kernel(const TpArgmaxParams p)
{
    __shared__ float s_v[8];
    __shared__ int s_i[8];
    pdl_launch_dependents();
    pdl_wait(); // the lm_head kernel's per-CTA results
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const unsigned E = *p.epoch + (unsigned)p.phase + 1u;
    float v = -INFINITY;
    int i = INT_MAX;
    for (int b = tid; b < p.n_parts; b += blockDim.x)
        better(v, i, __ldcg(p.part_val + b), __ldcg(p.part_idx + b));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        better(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
    if (lane == 0)
    {
        s_v[warp] = v;
        s_i[warp] = i;
    }
    __syncthreads();
    if (tid != 0)
        return;
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
        better(v, i, s_v[w], s_i[w]);
    // publish (value, index) in every rank's slot for this rank, then signal
    for (int q = 0; q < p.c.size; ++q)
    {
        volatile float* slot = reinterpret_cast<volatile float*>(p.c.best[q] + p.c.rank);
        slot[0] = v;
        slot[1] = __int_as_float(i);
    }
    tp_signal(p.c, E);
    float gv = -INFINITY;
    int gi = INT_MAX;
    if (tp_wait_flags(p.c, E, p.state))
        for (int w = 0; w < p.c.size; ++w)
        {
            volatile const float* slot = reinterpret_cast<volatile const float*>(p.c.best[p.c.rank] + w);
            better(gv, gi, slot[0], __float_as_int(slot[1]));
        }
    const uint32_t token = (gi == INT_MAX) ? 0u : (uint32_t)gi;
    DecodeState* st = p.state;
    const uint32_t pos = st->pos;
    if (pos + 1 >= st->n_prompt)
    {
        const uint32_t g = pos + 1 - st->n_prompt;
        if (g < (uint32_t)p.max_seq)
            p.out_tokens[g] = token;
    }
    st->next_token = token;
    st->pos = pos + 1;
    st->lm_counter = 0u;
}

// Advances the epoch by one step's worth (last kernel of every step graph).
__global__ void tp_epoch_kernel(unsigned* epoch, unsigned steps_phases)
{
    if (threadIdx.x == 0)
        *epoch += steps_phases;
}

} // namespace aaedn_dev
