// lwm_mppi.cuh — MPPI weighting as a one-pass, multi-block reduction.
//
// Reference: mppi_weighted_sequence (src/planner.rs:1588-1602) computes
//   w_s = softmax_s(-(score_s - min score) / lambda),  mean' = sum_s w_s cand_s
// and lowest_score_indices(scores, 1) (src/planner.rs:1647) the argmin with
// NaN ranked as +inf and ties to the lower index.
//
// Here every block reduces its own rows to a tuple
//   (m_p = local min, W_p = sum exp((s - m_p) * mul), V_p[e] = sum exp(..) cand[e],
//    key_p = smallest (score, index) key)
// with mul = -1/lambda, and the last block of a vehicle to arrive rescales the
// tuples by exp((m_p - M) * mul), M = global min, and writes mean' = V / W.
// exp((s-m_p)mul) * exp((m_p-M)mul) = exp((s-M)mul), so this equals the
// reference's softmax up to f32 rounding.
#pragma once

#include <cstdint>

#include "lwm_device.cuh"
#include "lwm_kernels.hpp"

namespace lwm {

// One element of the white-noise candidate sampler: candidate (b, s) of a
// plan with S samples per vehicle, step t, action act (of A; horizon T):
// slot 0 of the unsharded plan is the mean, the others mean + eps std with
// eps the injected noise or the Philox normal of the global index, then the
// action bounds (sample_candidates, src/planner.rs:1152-1208, 1614-1616).
__device__ __forceinline__ float sample_white(const float* mean, const float* std, const float* low,
                                             const float* high, const float* noise, uint64_t seed, uint64_t offset,
                                             uint32_t sample_base, uint32_t sample_total, uint32_t b, uint32_t s,
                                             uint32_t t, uint32_t act, uint32_t S, uint32_t T, uint32_t A) {
    const size_t mi = (static_cast<size_t>(b) * T + t) * A + act;
    float v;
    if (sample_base + s == 0) {
        v = mean[mi];
    } else {
        const uint64_t e = ((static_cast<uint64_t>(b) * S + s) * T + t) * A + act;
        const uint64_t gi = global_row(b, s, sample_base, sample_total, S) * T * A + static_cast<uint64_t>(t) * A + act;
        const float eps = noise ? noise[e] : normal_at(seed, offset + gi);
        v = __fadd_rn(mean[mi], __fmul_rn(eps, std[mi]));
    }
    return cmin(cmax(v, low[act]), high[act]);
}

template <int NT>
__device__ __forceinline__ uint64_t block_min_u64(uint64_t v, uint64_t* scratch) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const uint64_t o = __shfl_xor_sync(0xffffffffu, v, off);
        v = o < v ? o : v;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    uint64_t r = scratch[0];
#pragma unroll
    for (int w = 1; w < NT / 32; ++w) r = scratch[w] < r ? scratch[w] : r;
    return r;
}

template <int NT>
__device__ __forceinline__ float block_sum_f32(float v, float* scratch) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float r = 0.0f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) r += scratch[w];
    return r;
}

// Combines `count` tuples (stride `stride` floats apart, starting at `base`)
// of vehicle b into the final outputs, or into a.shard_tuple.  All NT threads
// call it.
template <int NT>
__device__ void mppi_finish(const MppiArgs& a, uint32_t b, const float* base, uint32_t count, size_t stride,
                            uint64_t* s_key_scratch) {
    const uint32_t TA = a.T * a.A;
    uint64_t gkey = ~0ull;
    // (the tuples were written by other blocks before their arrival on the
    // vehicle's counter: read at L2, where they are, with loads independent of
    // one another so that they overlap)
    for (uint32_t q = threadIdx.x; q < count; q += NT) {
        const uint64_t k = __ldcg(reinterpret_cast<const unsigned long long*>(base + static_cast<size_t>(q) * stride) + 1);
        gkey = k < gkey ? k : gkey;
    }
    gkey = block_min_u64<NT>(gkey, s_key_scratch);
    const float M = key_score(gkey);
    float* tuple = a.shard_tuple ? a.shard_tuple + static_cast<size_t>(b) * a.pw : nullptr;
    float Wtot = 0.0f;
    for (uint32_t e = threadIdx.x; e < TA; e += NT) {
        float W = 0.0f, V = 0.0f;
#pragma unroll 4
        for (uint32_t q = 0; q < count; ++q) {
            const float* pq = base + static_cast<size_t>(q) * stride;
            const uint64_t k = __ldcg(reinterpret_cast<const unsigned long long*>(pq) + 1);
            const float m = __ldcg(pq), w = __ldcg(pq + 1), v = __ldcg(pq + 4 + e);
            if (k == ~0ull) continue;  // tuple without rows
            const float f = expf((m - M) * a.mul);
            W += w * f;
            V += v * f;
        }
        Wtot = W;
        if (tuple) {
            tuple[4 + e] = V;
            continue;
        }
        const float value = V / W;
        const uint32_t t = e / a.A, act = e - t * a.A;
        const size_t seq = static_cast<size_t>(b) * TA;
        a.sequence[seq + e] = value;
        if (t == 0) a.first_action[static_cast<size_t>(b) * a.A + act] = value;
        if (t >= 1) a.warm_start[seq + e - a.A] = value;
        if (t == a.T - 1) a.warm_start[seq + e] = value;
    }
    if (threadIdx.x == 0) {
        if (tuple) {
            tuple[0] = M;
            tuple[1] = Wtot;
            reinterpret_cast<uint64_t*>(tuple)[1] = gkey;
        } else {
            a.best_index[b] = static_cast<uint32_t>(gkey & 0xffffffffu);
            a.best_score[b] = M;
        }
    }
}

// All NT threads of the block call this.  Rows r in [0, nrows) of this block
// have score s_score[r] (smem) and sample index first_sample + r; candidate
// element e of row r is cand[r * row_stride + e] (smem or global).  s_w is
// smem scratch of >= nrows floats.  Writes partial p of vehicle b and, if this
// block is the last of the vehicle, the final outputs.
template <int NT>
__device__ void mppi_reduce_rows(const MppiArgs& a, uint32_t b, uint32_t p, uint32_t nrows,
                                 const float* s_score, uint32_t first_sample, const float* cand,
                                 size_t row_stride, float* s_w) {
    __shared__ uint64_t s_key_scratch[NT / 32];
    __shared__ float s_f_scratch[NT / 32];
    __shared__ int s_is_last;
    const uint32_t TA = a.T * a.A;

    uint64_t key = ~0ull;
    for (uint32_t r = threadIdx.x; r < nrows; r += NT) {
        const uint64_t k = score_key(s_score[r], a.sample_base + first_sample + r);
        key = k < key ? k : key;
    }
    key = block_min_u64<NT>(key, s_key_scratch);
    const float m = key_score(key);
    float wsum = 0.0f;
    for (uint32_t r = threadIdx.x; r < nrows; r += NT) {
        const float w = expf((s_score[r] - m) * a.mul);
        s_w[r] = w;
        wsum += w;
    }
    wsum = block_sum_f32<NT>(wsum, s_f_scratch);  // contains __syncthreads: s_w visible
    float* part = a.partials + (static_cast<size_t>(b) * a.P + p) * a.pw;
    for (uint32_t e = threadIdx.x; e < TA; e += NT) {
        float acc = 0.0f;
        for (uint32_t r = 0; r < nrows; ++r) acc += s_w[r] * cand[r * row_stride + e];
        part[4 + e] = acc;
    }
    if (threadIdx.x == 0) {
        part[0] = m;
        part[1] = wsum;
        reinterpret_cast<uint64_t*>(part)[1] = key;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int done = atomicAdd(&a.counters[b], 1u);
        s_is_last = (done == a.P - 1) ? 1 : 0;
    }
    __syncthreads();
    if (!s_is_last) return;
    __threadfence();

    mppi_finish<NT>(a, b, a.partials + static_cast<size_t>(b) * a.P * a.pw, a.P, a.pw, s_key_scratch);
    if (threadIdx.x == 0) a.counters[b] = 0u;
}

}  // namespace lwm
