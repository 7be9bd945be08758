// kernels_planner.cu — the planner's own kernels (sampling, MPPI reduction,
// top-k elite selection and refit, colored noise), used by CEM / iCEM and by
// MPPI with a caller-supplied scorer.  The built-in scorers fuse sampling and
// the MPPI reduction into their rollout kernels instead (kernels_nominal.cu,
// kernels_skyjepa.cu).
#include <algorithm>
#include <cstdint>
#include <mutex>

#include "lwm_device.cuh"
#include "lwm_kernels.hpp"
#include "lwm_mppi.cuh"

namespace lwm {

// color_temporal_noise of one (sample, action) lane held in registers
// (swm_temporal_color_noise_f32, src/planner.rs:1852-1896): EMA with factor
// `smooth`, then centre and scale by 1 / sqrt(var + 1e-6) over the horizon.
__device__ __forceinline__ void color_lane(float (&eps)[kMaxHorizon], uint32_t T, float smooth) {
    const float keep = 1.0f - smooth;
    float prev = eps[0], mean = 0.0f;
    for (uint32_t t = 0; t < T; ++t) {
        prev = (t == 0) ? eps[t] : fmaf(smooth, prev, keep * eps[t]);
        eps[t] = prev;
        mean += prev;
    }
    mean /= static_cast<float>(T);
    float var = 0.0f;
    for (uint32_t t = 0; t < T; ++t) {
        const float c = eps[t] - mean;
        eps[t] = c;
        var += c * c;
    }
    const float inv_std = 1.0f / sqrtf(var / static_cast<float>(T) + 1.0e-6f);
    for (uint32_t t = 0; t < T; ++t) eps[t] *= inv_std;
}

// ----------------------------------------------------------------- sampling
//
// One thread per (vehicle, sample, action) lane over the horizon:
//   sample_candidates / sample_candidates_with_temporal_noise
//   (src/planner.rs:1152-1196): eps ~ N(0,1) (injected or Philox), optional
//   colored-noise EMA + standardisation (:1516-1586, kernel :1852-1896),
//   cand = mean + eps*std, slot 0 = mean (:1198-1208), clamp (:1614-1616),
//   then inject_carried_elites (:1210-1235) into slots 1..1+inject.
__global__ void __launch_bounds__(256) sample_kernel(SampleArgs a) {
    const uint64_t lane_id = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint64_t lanes = static_cast<uint64_t>(a.B) * a.S * a.A;
    if (lane_id >= lanes) return;
    const uint32_t act = static_cast<uint32_t>(lane_id % a.A);
    const uint64_t row = lane_id / a.A;  // b * S + s
    const uint32_t s = static_cast<uint32_t>(row % a.S);
    const uint32_t b = static_cast<uint32_t>(row / a.S);
    const uint64_t base = row * a.T * a.A + act;
    const uint64_t gbase = global_row(b, s, a.sample_base, a.sample_total, a.S) * a.T * a.A + act;
    float eps[kMaxHorizon];
    for (uint32_t t = 0; t < a.T; ++t) {
        const uint64_t idx = base + static_cast<uint64_t>(t) * a.A;
        eps[t] = a.noise ? a.noise[idx] : normal_at(a.seed, a.offset + gbase + static_cast<uint64_t>(t) * a.A);
    }
    if (a.smooth > 0.0f && a.T > 1) color_lane(eps, a.T, a.smooth);
    const uint32_t g = a.sample_base + s;  // the candidate's row in the (unsharded) plan
    const bool carried = a.carried && g >= 1 && g <= a.inject;
    const float lo = a.low[act], hi = a.high[act];
    for (uint32_t t = 0; t < a.T; ++t) {
        const size_t mi = (static_cast<size_t>(b) * a.T + t) * a.A + act;
        float v;
        if (carried) {
            v = a.carried[((static_cast<size_t>(b) * a.carried_count + (g - 1)) * a.T + t) * a.A + act];
        } else {
            v = (a.sample_base + s == 0) ? a.mean[mi] : __fadd_rn(a.mean[mi], __fmul_rn(eps[t], a.std[mi]));
            v = cmin(cmax(v, lo), hi);
        }
        a.out[base + static_cast<uint64_t>(t) * a.A] = v;
    }
}

// The same without the colored-noise pass (white noise): one thread per
// (vehicle, sample, step, action) element, each of which is independent.
__global__ void __launch_bounds__(256) sample_elem_kernel(SampleArgs a) {
    const uint64_t e = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint32_t TA = a.T * a.A;
    if (e >= static_cast<uint64_t>(a.B) * a.S * TA) return;
    const uint32_t act = static_cast<uint32_t>(e % a.A);
    const uint32_t t = static_cast<uint32_t>((e / a.A) % a.T);
    const uint64_t row = e / TA;  // b * S + s
    const uint32_t s = static_cast<uint32_t>(row % a.S);
    const uint32_t b = static_cast<uint32_t>(row / a.S);
    const uint32_t g = a.sample_base + s;  // the candidate's row in the (unsharded) plan
    float v;
    if (a.carried && g >= 1 && g <= a.inject)
        v = a.carried[((static_cast<size_t>(b) * a.carried_count + (g - 1)) * a.T + t) * a.A + act];
    else
        v = sample_white(a.mean, a.std, a.low, a.high, a.noise, a.seed, a.offset, a.sample_base, a.sample_total, b, s,
                         t, act, a.S, a.T, a.A);
    a.out[e] = v;
}

// The same for 4 consecutive actions per thread (A a multiple of 4, the
// stream offset too): the 4 draws of one step come from one Philox block,
// so each block is evaluated once, and the row is stored as one float4.
__global__ void __launch_bounds__(256) sample_quad_kernel(SampleArgs a) {
    const uint64_t q = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const uint32_t TA = a.T * a.A;
    if (q >= static_cast<uint64_t>(a.B) * a.S * TA / 4) return;
    const uint64_t e = q * 4;
    const uint32_t act = static_cast<uint32_t>(e % a.A);
    const uint32_t t = static_cast<uint32_t>((e / a.A) % a.T);
    const uint64_t row = e / TA;  // b * S + s
    const uint32_t s = static_cast<uint32_t>(row % a.S);
    const uint32_t b = static_cast<uint32_t>(row / a.S);
    const uint32_t g = a.sample_base + s;
    float v[4];
    if (a.carried && g >= 1 && g <= a.inject) {
        const float* src = a.carried + ((static_cast<size_t>(b) * a.carried_count + (g - 1)) * a.T + t) * a.A + act;
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = src[i];
    } else {
        const size_t mi = (static_cast<size_t>(b) * a.T + t) * a.A + act;
        if (g == 0) {
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = a.mean[mi + i];
        } else {
            float eps[4];
            if (a.noise) {
#pragma unroll
                for (int i = 0; i < 4; ++i) eps[i] = a.noise[e + i];
            } else {
                const uint64_t gi = global_row(b, s, a.sample_base, a.sample_total, a.S) * TA +
                                    static_cast<uint64_t>(t) * a.A + act;
                const float4 n = normal_quad(a.seed, (a.offset + gi) >> 2);
                eps[0] = n.x; eps[1] = n.y; eps[2] = n.z; eps[3] = n.w;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = __fadd_rn(a.mean[mi + i], __fmul_rn(eps[i], a.std[mi + i]));
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = cmin(cmax(v[i], a.low[act + i]), a.high[act + i]);
    }
    *reinterpret_cast<float4*>(a.out + e) = make_float4(v[0], v[1], v[2], v[3]);
}

// --------------------------------------------------- MPPI reduce (generic)
__global__ void __launch_bounds__(256) mppi_reduce_kernel(MppiArgs m, const float* cand,
                                                          const float* scores, uint32_t S) {
    constexpr int NT = 256;
    __shared__ float s_score[NT];
    __shared__ float s_w[NT];
    const uint32_t b = blockIdx.y, p = blockIdx.x;
    const uint32_t first = p * NT;
    const uint32_t nrows = min(static_cast<uint32_t>(NT), S - first);
    if (threadIdx.x < nrows) s_score[threadIdx.x] = scores[static_cast<size_t>(b) * S + first + threadIdx.x];
    __syncthreads();
    const size_t TA = static_cast<size_t>(m.T) * m.A;
    mppi_reduce_rows<NT>(m, b, p, nrows, s_score, first,
                         cand + (static_cast<size_t>(b) * S + first) * TA, TA, s_w);
}

// ------------------------------------------- MPPI combine across shards
// One block per vehicle: the tuples of every candidate-range shard
// ([shards][B][pw], gathered from the GPUs that scored them) are rescaled to
// the global minimum and summed, exactly as the per-block partials are.
__global__ void __launch_bounds__(256) mppi_combine_kernel(MppiArgs m, const float* tuples, uint32_t B,
                                                           uint32_t shards) {
    __shared__ uint64_t s_key_scratch[256 / 32];
    const uint32_t b = blockIdx.x;
    mppi_finish<256>(m, b, tuples + static_cast<size_t>(b) * m.pw, shards, static_cast<size_t>(B) * m.pw,
                     s_key_scratch);
}

// ------------------------------------------------ top-k + elite refit
//
// One block per vehicle.  lowest_score_indices (src/planner.rs:1647-1659:
// ascending scores, NaN as +inf, ties to the lower index) is the ascending
// order of the unique 64-bit keys (score, index).  Short rows are sorted
// whole in shared memory (bitonic).  Longer rows are radix-selected first:
// four 8-bit digit passes over the scores find the K-th smallest score, an
// ordered compaction keeps the keys below it and the lowest-index keys equal
// to it (exactly K keys), and only those K are sorted — the same K keys in
// the same order as the full sort, with no limit on the row length.  Then
// select_elites + gather_candidate_sequences (:1730-1754) and the refit of
//   CEM  (:516-517):  mean = elites.mean(1), std = max(sqrt(var_unbiased), min_std)
//   iCEM (:859-868):  mean = momentum(mean, elite_mean, alpha),
//                     std = max(momentum(std, max(sqrt(var), min_std), alpha), min_std)
// plus carried elites (:869-873), the best index and the returned sequence.
__device__ __forceinline__ void bitonic_sort_keys(uint64_t* keys, uint32_t n) {
    for (uint32_t width = 2; width <= n; width <<= 1) {
        for (uint32_t stride = width >> 1; stride > 0; stride >>= 1) {
            for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
                const uint32_t peer = i ^ stride;
                if (peer > i) {
                    const uint64_t x = keys[i], y = keys[peer];
                    const bool ascending = (i & width) == 0;
                    if ((x > y) == ascending) {
                        keys[i] = y;
                        keys[peer] = x;
                    }
                }
            }
            __syncthreads();
        }
    }
}

// The orderable score word of score_key (its high 32 bits).
__device__ __forceinline__ uint32_t score_ord(float v) { return static_cast<uint32_t>(score_key(v, 0u) >> 32); }

struct SelectShared {
    uint32_t hist[256];
    uint32_t warp_lt[32], warp_eq[32];
    uint32_t bin, need;
};

// keys[0..K) = the K lowest keys of scores[0..S) in ascending order; keys has
// room for `len` entries (sort_length(S) for a whole-row sort, else
// sort_length(K)).  Needs blockDim.x a multiple of 32, at most 1024, and
// 1 <= K <= S.
__device__ void lowest_keys(const float* scores, uint32_t S, uint32_t K, uint32_t len, bool select,
                            uint64_t* keys) {
    const uint32_t tid = threadIdx.x, nt = blockDim.x, lane = tid & 31u, warp = tid >> 5, nwarps = nt >> 5;
    if (!select) {
        for (uint32_t i = tid; i < len; i += nt) keys[i] = i < S ? score_key(scores[i], i) : ~0ull;
        __syncthreads();
        bitonic_sort_keys(keys, len);
        return;
    }
    __shared__ SelectShared sh;
    // 1. the K-th smallest score word, one 8-bit digit per pass (most significant first)
    uint32_t prefix = 0u, mask = 0u, need = K;  // need: rank of the K-th key inside the current bucket
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (uint32_t i = tid; i < 256; i += nt) sh.hist[i] = 0u;
        __syncthreads();
        for (uint32_t base = 0; base < S; base += nt) {  // block-uniform trip count: whole warps below
            const uint32_t i = base + tid;
            bool take = false;
            uint32_t bin = 256u + lane;  // lanes that do not count get a bin of their own
            if (i < S) {
                const uint32_t o = score_ord(scores[i]);
                take = (o & mask) == prefix;
                if (take) bin = (o >> shift) & 255u;
            }
            const uint32_t peers = __match_any_sync(0xffffffffu, bin);
            if (take && lane == static_cast<uint32_t>(__ffs(peers) - 1)) atomicAdd(&sh.hist[bin], __popc(peers));
        }
        if (tid == 0) {  // overwritten below; keeps the state defined whatever the counts
            sh.bin = 0u;
            sh.need = need;
        }
        __syncthreads();
        if (warp == 0) {
            uint32_t c[8], sum = 0u;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                c[j] = sh.hist[lane * 8u + j];
                sum += c[j];
            }
            uint32_t incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= static_cast<uint32_t>(o)) incl += v;
            }
            uint32_t run = incl - sum;
            if (run < need && need <= incl) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (run < need && need <= run + c[j]) {
                        sh.bin = lane * 8u + j;
                        sh.need = need - run;
                    }
                    run += c[j];
                }
            }
        }
        __syncthreads();
        prefix |= sh.bin << shift;
        mask |= 255u << shift;
        need = sh.need;
        __syncthreads();
    }
    // 2. ordered compaction: every key below the K-th score word, then the
    //    `need` lowest-index keys equal to it
    const uint32_t n_less = K - need;
    const uint32_t below = (1u << lane) - 1u;
    uint32_t lt_base = 0u, eq_base = 0u;
    for (uint32_t base = 0; base < S; base += nt) {
        const uint32_t i = base + tid;
        uint32_t o = 0u;
        bool lt = false, eq = false;
        if (i < S) {
            o = score_ord(scores[i]);
            lt = o < prefix;
            eq = o == prefix;
        }
        const uint32_t blt = __ballot_sync(0xffffffffu, lt), beq = __ballot_sync(0xffffffffu, eq);
        if (lane == 0) {
            sh.warp_lt[warp] = __popc(blt);
            sh.warp_eq[warp] = __popc(beq);
        }
        __syncthreads();
        uint32_t off_lt = 0u, off_eq = 0u, tot_lt = 0u, tot_eq = 0u;
        for (uint32_t w = 0; w < nwarps; ++w) {
            const uint32_t nl = sh.warp_lt[w], ne = sh.warp_eq[w];
            if (w < warp) {
                off_lt += nl;
                off_eq += ne;
            }
            tot_lt += nl;
            tot_eq += ne;
        }
        const uint64_t key = (static_cast<uint64_t>(o) << 32) | i;
        if (lt) {
            const uint32_t r = lt_base + off_lt + __popc(blt & below);
            if (r < n_less) keys[r] = key;  // always true: exactly n_less keys are below
        }
        if (eq) {
            const uint32_t r = eq_base + off_eq + __popc(beq & below);
            if (r < need) keys[n_less + r] = key;
        }
        lt_base += tot_lt;
        eq_base += tot_eq;
        __syncthreads();
        if (lt_base == n_less && eq_base >= need) break;  // block-uniform: every key is placed
    }
    for (uint32_t i = K + tid; i < len; i += nt) keys[i] = ~0ull;
    __syncthreads();
    bitonic_sort_keys(keys, len);
}

__global__ void __launch_bounds__(1024) topk_refit_kernel(RefitArgs a) {
    extern __shared__ uint64_t s_keys[];
    const uint32_t b = blockIdx.x;
    lowest_keys(a.scores + static_cast<size_t>(b) * a.S, a.S, a.K, a.sort_len, a.select != 0, s_keys);
    const uint32_t TA = a.T * a.A;
    const size_t seq = static_cast<size_t>(b) * TA;
    const float* cb = a.cand + static_cast<size_t>(b) * a.S * TA;
    const uint32_t* imap = a.index_map ? a.index_map + static_cast<size_t>(b) * a.S : nullptr;
    if (a.elite_index)
        for (uint32_t j = threadIdx.x; j < a.K; j += blockDim.x) {
            const uint32_t i = static_cast<uint32_t>(s_keys[j]);
            a.elite_index[static_cast<size_t>(b) * a.K + j] = imap ? imap[i] : i;
        }
    const float inv_k = a.inv_k, inv_km1 = a.inv_km1;
    const uint32_t best = static_cast<uint32_t>(s_keys[0]);
    for (uint32_t e = threadIdx.x; e < TA; e += blockDim.x) {
        float sum = 0.0f;
        for (uint32_t j = 0; j < a.K; ++j) sum += cb[static_cast<size_t>(static_cast<uint32_t>(s_keys[j])) * TA + e];
        const float m = sum * inv_k;
        float sq = 0.0f;
        for (uint32_t j = 0; j < a.K; ++j) {
            const float d = cb[static_cast<size_t>(static_cast<uint32_t>(s_keys[j])) * TA + e] - m;
            sq += d * d;
        }
        float sd = sqrtf(sq * inv_km1);
        if (a.min_std != 0.0f) sd = cmax(sd, a.min_std);
        if (a.elite_mean_out) a.elite_mean_out[seq + e] = m;
        float new_mean = m, new_std = sd;
        if (a.icem) {
            const float pm = a.mean[seq + e], ps = a.std[seq + e];
            if (a.alpha == 0.0f) {
                new_mean = m; new_std = sd;
            } else if (a.alpha == 1.0f) {
                new_mean = pm; new_std = ps;
            } else {
                const float beta = 1.0f - a.alpha;
                new_mean = __fadd_rn(__fmul_rn(pm, a.alpha), __fmul_rn(m, beta));
                new_std = __fadd_rn(__fmul_rn(ps, a.alpha), __fmul_rn(sd, beta));
            }
            if (a.min_std != 0.0f) new_std = cmax(new_std, a.min_std);
        }
        a.mean[seq + e] = new_mean;
        a.std[seq + e] = new_std;
        for (uint32_t j = 0; j < a.keep; ++j)
            a.carried[(static_cast<size_t>(b) * a.keep + j) * TA + e] =
                cb[static_cast<size_t>(static_cast<uint32_t>(s_keys[j])) * TA + e];
        const float out = a.return_best ? cb[static_cast<size_t>(best) * TA + e] : new_mean;
        const uint32_t t = e / a.A, act = e - t * a.A;
        a.sequence[seq + e] = out;
        if (t == 0) a.first_action[static_cast<size_t>(b) * a.A + act] = out;
        if (a.warm_start) {
            if (t >= 1) a.warm_start[seq + e - a.A] = out;
            if (t == a.T - 1) a.warm_start[seq + e] = out;
        }
    }
    if (threadIdx.x == 0) {
        a.best_index[b] = imap ? imap[best] : best;
        a.best_score[b] = key_score(s_keys[0]);
    }
}

// ------------------------------------------ candidate shards of CEM / iCEM
//
// A shard's lowest `K` candidates (the order of lowest_score_indices) as
// tuples [B][K][2 + T*A]: score, global candidate index (bits), actions.
// The union of every shard's tuples holds the plan's global elites, and
// sorting the union by (score, position) with positions in shard order gives
// the (score, global index) order of the unsharded selection.
__global__ void __launch_bounds__(1024) elite_tuples_kernel(const float* scores, const float* cand, uint32_t S,
                                                            uint32_t sort_len, uint32_t select, uint32_t K,
                                                            uint32_t TA, uint32_t base, float* out) {
    extern __shared__ uint64_t s_keys[];
    const uint32_t b = blockIdx.x, W = 2 + TA;
    lowest_keys(scores + static_cast<size_t>(b) * S, S, K, sort_len, select != 0, s_keys);
    for (uint32_t q = threadIdx.x; q < K * W; q += blockDim.x) {
        const uint32_t j = q / W, f = q % W, idx = static_cast<uint32_t>(s_keys[j]);
        const size_t row = static_cast<size_t>(b) * S + idx;
        const float v = f == 0 ? scores[row] : (f == 1 ? __uint_as_float(base + idx) : cand[row * TA + f - 2]);
        out[(static_cast<size_t>(b) * K + j) * W + f] = v;
    }
}

// gathered [G][B][K][W] (shard-major) -> merged scores [B][G*K], candidates
// [B][G*K][T*A] and global indices [B][G*K].
__global__ void __launch_bounds__(256) elite_merge_kernel(const float* gathered, uint32_t G, uint32_t B, uint32_t K,
                                                          uint32_t TA, float* scores, float* cand, uint32_t* index) {
    const uint32_t W = 2 + TA;
    const uint64_t total = static_cast<uint64_t>(G) * B * K * W;
    for (uint64_t e = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t f = static_cast<uint32_t>(e % W);
        uint64_t r = e / W;
        const uint32_t k = static_cast<uint32_t>(r % K);
        r /= K;
        const uint32_t b = static_cast<uint32_t>(r % B), sh = static_cast<uint32_t>(r / B);
        const size_t m = static_cast<size_t>(b) * G * K + static_cast<size_t>(sh) * K + k;
        const float v = gathered[e];
        if (f == 0) scores[m] = v;
        else if (f == 1) index[m] = __float_as_uint(v);
        else cand[m * TA + f - 2] = v;
    }
}

// lowest_score_indices alone (the swm_lowest_k_indices_f32 replacement).
__global__ void __launch_bounds__(1024) lowest_k_kernel(const float* scores, uint32_t* out, uint32_t S,
                                                        uint32_t sort_len, uint32_t select, uint32_t K) {
    extern __shared__ uint64_t s_keys[];
    const uint32_t b = blockIdx.x;
    lowest_keys(scores + static_cast<size_t>(b) * S, S, K, sort_len, select != 0, s_keys);
    for (uint32_t j = threadIdx.x; j < K; j += blockDim.x)
        out[static_cast<size_t>(b) * K + j] = static_cast<uint32_t>(s_keys[j]);
}

// color_temporal_noise alone: each thread loads one (sample, action) lane
// into registers, colors it with the sampler's lane code and stores it.
__global__ void __launch_bounds__(256) color_noise_kernel(const float* in, float* out, uint64_t lanes, uint32_t T,
                                                          uint32_t A, float smooth) {
    const uint64_t lane_id = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (lane_id >= lanes) return;
    const uint64_t row = lane_id / A;
    const uint32_t act = static_cast<uint32_t>(lane_id - row * A);
    const float* src = in + row * T * A + act;
    float eps[kMaxHorizon];
    for (uint32_t t = 0; t < T; ++t) eps[t] = src[static_cast<size_t>(t) * A];
    color_lane(eps, T, smooth);
    float* dst = out + row * T * A + act;
    for (uint32_t t = 0; t < T; ++t) dst[static_cast<size_t>(t) * A] = eps[t];
}

__global__ void __launch_bounds__(256) normal_fill_kernel(uint64_t seed, uint64_t offset, uint64_t count,
                                                          float* out) {
    const uint64_t i = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < count) out[i] = normal_at(seed, offset + i);
}

// ----------------------------------------------------------------- launchers

static inline uint32_t ceil_div(uint64_t a, uint64_t b) { return static_cast<uint32_t>((a + b - 1) / b); }

cudaError_t launch_sample(const SampleArgs& a, cudaStream_t stream) {
    const uint64_t lanes = static_cast<uint64_t>(a.B) * a.S * a.A;
    if (a.smooth > 0.0f && a.T > 1)
        sample_kernel<<<ceil_div(lanes, 256), 256, 0, stream>>>(a);
    else if (a.A % 4 == 0 && a.offset % 4 == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15u) == 0)
        sample_quad_kernel<<<ceil_div(lanes * a.T / 4, 256), 256, 0, stream>>>(a);
    else
        sample_elem_kernel<<<ceil_div(lanes * a.T, 256), 256, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_mppi_reduce(const MppiArgs& m, const float* cand, const float* scores, uint32_t B,
                               uint32_t S, cudaStream_t stream) {
    dim3 grid(ceil_div(S, 256), B);
    mppi_reduce_kernel<<<grid, 256, 0, stream>>>(m, cand, scores, S);
    return cudaGetLastError();
}

cudaError_t launch_mppi_combine(const MppiArgs& m, const float* tuples, uint32_t B, uint32_t shards,
                                cudaStream_t stream) {
    MppiArgs mm = m;
    mm.shard_tuple = nullptr;
    mppi_combine_kernel<<<B, 256, 0, stream>>>(mm, tuples, B, shards);
    return cudaGetLastError();
}

uint32_t sort_length(uint32_t S) {
    uint32_t n = 1;
    while (n < S) n <<= 1;
    return n;
}

bool topk_layout(uint32_t S, uint32_t K, uint32_t* len, uint32_t* select) {
    if (K == 0 || K > S || K > kMaxElites) return false;
    const bool sel = S > kSortWholeRow;
    *select = sel ? 1u : 0u;
    *len = sort_length(sel ? K : S);
    return true;
}

namespace {

// Dynamic shared memory for `len` keys, with the opt-in above 48 KB made
// once per (kernel, device) for the largest layout.
template <typename Kern>
cudaError_t keys_smem(Kern kernel, uint32_t len, size_t* smem) {
    *smem = static_cast<size_t>(len) * sizeof(uint64_t);
    if (*smem <= 48 * 1024) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    static std::mutex mu;
    static bool done[3][64] = {};
    const int which = reinterpret_cast<const void*>(kernel) == reinterpret_cast<const void*>(topk_refit_kernel) ? 0
                      : reinterpret_cast<const void*>(kernel) == reinterpret_cast<const void*>(elite_tuples_kernel) ? 1
                                                                                                                  : 2;
    std::lock_guard<std::mutex> lock(mu);
    if (!done[which][dev]) {
        const size_t max_smem = static_cast<size_t>(sort_length(kMaxElites > kSortWholeRow ? kMaxElites : kSortWholeRow)) *
                                sizeof(uint64_t);
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(max_smem));
        if (e != cudaSuccess) return e;
        done[which][dev] = true;
    }
    return cudaSuccess;
}

uint32_t keys_threads(uint32_t len, uint32_t select) {
    if (select) return 1024;  // the selection passes stride the whole row
    return len < 1024 ? (len < 64 ? 64 : len) : 1024;
}

}  // namespace

cudaError_t launch_topk_refit(const RefitArgs& a, uint32_t B, cudaStream_t stream) {
    size_t smem = 0;
    cudaError_t e = keys_smem(topk_refit_kernel, a.sort_len, &smem);
    if (e != cudaSuccess) return e;
    topk_refit_kernel<<<B, keys_threads(a.sort_len, a.select), smem, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_elite_tuples(const float* scores, const float* cand, uint32_t B, uint32_t S, uint32_t K,
                                uint32_t TA, uint32_t base, float* out, cudaStream_t stream) {
    uint32_t len = 0, select = 0;
    if (!topk_layout(S, K, &len, &select)) return cudaErrorInvalidValue;
    size_t smem = 0;
    cudaError_t e = keys_smem(elite_tuples_kernel, len, &smem);
    if (e != cudaSuccess) return e;
    elite_tuples_kernel<<<B, 1024, smem, stream>>>(scores, cand, S, len, select, K, TA, base, out);
    return cudaGetLastError();
}

cudaError_t launch_elite_merge(const float* gathered, uint32_t G, uint32_t B, uint32_t K, uint32_t TA, float* scores,
                               float* cand, uint32_t* index, cudaStream_t stream) {
    const uint64_t total = static_cast<uint64_t>(G) * B * K * (2 + TA);
    const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((total + 255) / 256, 148 * 16));
    elite_merge_kernel<<<blocks, 256, 0, stream>>>(gathered, G, B, K, TA, scores, cand, index);
    return cudaGetLastError();
}

cudaError_t launch_lowest_k(const float* scores, uint32_t* out, uint32_t B, uint32_t S, uint32_t K,
                            cudaStream_t stream) {
    uint32_t len = 0, select = 0;
    if (!topk_layout(S, K, &len, &select)) return cudaErrorInvalidValue;
    size_t smem = 0;
    cudaError_t e = keys_smem(lowest_k_kernel, len, &smem);
    if (e != cudaSuccess) return e;
    lowest_k_kernel<<<B, keys_threads(len, select), smem, stream>>>(scores, out, S, len, select, K);
    return cudaGetLastError();
}

cudaError_t launch_color_noise(const float* in, float* out, uint32_t B, uint32_t S, uint32_t T, uint32_t A,
                               float smooth, cudaStream_t stream) {
    const uint64_t seqs = static_cast<uint64_t>(B) * S * A;
    color_noise_kernel<<<ceil_div(seqs, 256), 256, 0, stream>>>(in, out, seqs, T, A, smooth);
    return cudaGetLastError();
}

cudaError_t launch_normal_fill(uint64_t seed, uint64_t offset, uint64_t count, float* out, cudaStream_t stream) {
    normal_fill_kernel<<<ceil_div(count, 256), 256, 0, stream>>>(seed, offset, count, out);
    return cudaGetLastError();
}

}  // namespace lwm
