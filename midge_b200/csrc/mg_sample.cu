// mg_sample.cu -- temperature / top-p sampling on the device
// (engine/midge.c:642-678 restated for one CTA per logits row).
//
// The reference softmaxes the logits with the temperature (float expf,
// double denominator), sorts (probability, index) descending, keeps the
// shortest prefix whose double running sum reaches top_p, draws
// r = u * sum(prefix) from its xorshift64* generator and walks the prefix
// until the running sum reaches r (the prefix's last entry when it never
// does).  Sorting 201,088 entries is the expensive part; here nothing is
// sorted.  Probabilities are >= 0, so their bit patterns order like their
// values, and both cut points -- where the sorted running mass reaches top_p
// and where it reaches r -- are found by a radix search over the bit
// patterns: three histogram passes (11 + 11 + 10 bits) of masses over the row,
// each narrowing to the one bin the running mass crosses, then, among the
// entries of exactly that probability, a count in index order.  Masses are
// summed as 2^-62 fixed point with integer atomics (the same result in every
// run); the reference sums the same values in double in sorted order, which
// differs by a few parts in 1e16.  Entries of exactly equal probability are
// taken in ascending index order (the reference's qsort leaves their order to
// the C library).  temp <= 0 is the greedy branch: the first maximum
// (engine/midge.c:655-660).
#include "mg_common.cuh"
#include "mg_kernels.h"

namespace mg {

constexpr int SP_THREADS = 1024;
constexpr int SP_BINS = 2048;
constexpr double SP_FIX = 4611686018427387904.0;  // 2^62

__device__ __forceinline__ unsigned long long sp_fix(float p) { return (unsigned long long)((double)p * SP_FIX); }

// xorshift64* draw as rng_u32 / rng_f of the reference (engine/midge.c:642-647)
__device__ __forceinline__ float sp_rng_f(uint64_t &st) {
    st ^= st >> 12;
    st ^= st << 25;
    st ^= st >> 27;
    const uint32_t u = (uint32_t)((st * 0x2545F4914F6CDD1DULL) >> 32);
    return (float)(u >> 8) / 16777216.0f;
}

struct SpSmem {
    unsigned long long mass[SP_BINS];
    unsigned cnt[SP_BINS];
    double dscr[32];
    unsigned long long uscr[32];
    long long lscr[32];
    float fscr[32];
    int iscr[32];
    uint32_t key;              // probability bits the search ended on
    unsigned long long above;  // fixed-point mass of the eligible entries above `key`
    unsigned ties;             // eligible entries with bits == key
    int found;
    long long pos;
};

template <typename T, typename Op>
__device__ T sp_reduce(T v, T *scratch, Op op) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) scratch[wid] = v;
    __syncthreads();
    if (wid == 0) {
        v = lane < (int)(blockDim.x >> 5) ? scratch[lane] : scratch[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) scratch[0] = v;
    }
    __syncthreads();
    v = scratch[0];
    __syncthreads();
    return v;
}

// Eligible entries: bits > fkey, or bits == fkey with index < flim.  Finds
// the bits K at which the descending running mass of the eligible entries
// reaches target: mass(> K) < target <= mass(>= K).  sm.found = 0 when their
// whole mass stays below target.
__device__ void sp_search(const float *pr, int64_t V, unsigned long long target, uint32_t fkey, int64_t flim,
                          SpSmem &sm) {
    uint32_t prefix = 0, pmask = 0;
    unsigned long long above = 0;
    for (int pass = 0; pass < 3; pass++) {
        const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
        const int nb = pass == 2 ? 1024 : 2048;
        for (int b = threadIdx.x; b < nb; b += blockDim.x) { sm.cnt[b] = 0; sm.mass[b] = 0; }
        __syncthreads();
        for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
            const float p = pr[i];
            const uint32_t key = __float_as_uint(p);
            if ((key > fkey || (key == fkey && i < flim)) && (key & pmask) == prefix) {
                const int b = (key >> shift) & (nb - 1);
                atomicAdd(&sm.mass[b], sp_fix(p));
                atomicAdd(&sm.cnt[b], 1u);
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int chosen = -1;
            for (int b = nb - 1; b >= 0; b--) {
                if (sm.cnt[b] && above + sm.mass[b] >= target) { chosen = b; break; }
                above += sm.mass[b];
            }
            sm.found = chosen >= 0;
            if (chosen >= 0) {
                prefix |= (uint32_t)chosen << shift;
                sm.ties = sm.cnt[chosen];
            }
            sm.key = prefix;
            sm.above = above;
        }
        __syncthreads();
        if (!sm.found) return;
        prefix = sm.key;
        above = sm.above;
        pmask |= (uint32_t)(nb - 1) << shift;
    }
}

// index of the t-th (0-based, index order) entry with bits == key and index
// < lim; -1 when there are not that many
__device__ long long sp_nth_equal(const float *pr, int64_t V, uint32_t key, int64_t lim, long long t, SpSmem &sm) {
    const int64_t per = (V + blockDim.x - 1) / blockDim.x;
    const int64_t a = (int64_t)threadIdx.x * per, b = min(V, a + per);
    int c = 0;
    for (int64_t i = a; i < b; i++) c += (__float_as_uint(pr[i]) == key && i < lim);
    int incl = c;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    __syncthreads();
    if (lane == 31) sm.iscr[wid] = incl;
    if (threadIdx.x == 0) sm.pos = -1;
    __syncthreads();
    if (wid == 0) {
        const int nw = blockDim.x >> 5;
        const int orig = lane < nw ? sm.iscr[lane] : 0;
        int x = orig;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += v;
        }
        if (lane < nw) sm.iscr[lane] = x - orig;
    }
    __syncthreads();
    const long long before = sm.iscr[wid] + incl - c;
    if (t >= before && t < before + c) {
        long long k = before;
        for (int64_t i = a; i < b; i++)
            if (__float_as_uint(pr[i]) == key && i < lim) {
                if (k == t) { sm.pos = i; break; }
                k++;
            }
    }
    __syncthreads();
    const long long r = sm.pos;
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(SP_THREADS)
    k_sample_topp(const float *__restrict__ logits, int64_t ldl, int64_t V, float temp, float topp,
                  uint64_t *__restrict__ rng, int32_t *__restrict__ out, float *__restrict__ probs) {
    extern __shared__ __align__(16) uint8_t sp_raw[];
    SpSmem &sm = *reinterpret_cast<SpSmem *>(sp_raw);
    const int row = blockIdx.x;
    const float *lg = logits + (int64_t)row * ldl;
    const float l0 = lg[0];
    // the maximum with the reference's strict > from element 0: NaN never
    // replaces a value, the first maximum wins, a NaN at element 0 stays
    float mx = -INFINITY;
    long long mi = V;
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = lg[i];
        if (v > mx) { mx = v; mi = i; }
    }
    const float gmx = sp_reduce(mx, sm.fscr, [](float a, float b) { return fmaxf(a, b); });
    long long cand = (mx == gmx) ? mi : (long long)V;
    cand = sp_reduce(cand, sm.lscr, [](long long a, long long b) { return a < b ? a : b; });
    if (temp <= 0.f) {
        if (threadIdx.x == 0) out[row] = (isnan(l0) || cand >= V) ? 0 : (int32_t)cand;
        return;
    }
    const float m0 = isnan(l0) ? l0 : gmx;
    float *pr = probs + (int64_t)row * V;
    double den = 0.0;
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
        const float p = expf(__fdiv_rn(__fsub_rn(lg[i], m0), temp));
        pr[i] = p;
        den += (double)p;
    }
    den = sp_reduce(den, sm.dscr, [](double a, double b) { return a + b; });
    const float fden = (float)den;
    for (int64_t i = threadIdx.x; i < V; i += blockDim.x) pr[i] = __fdiv_rn(pr[i], fden);
    __syncthreads();

    // the nucleus: the sorted prefix whose running mass first reaches top_p
    const double tp = (double)topp;
    const unsigned long long tfix = tp <= 0.0 ? 1ull : (tp >= 2.0 ? ~0ull : (unsigned long long)(tp * SP_FIX));
    sp_search(pr, V, tfix, 0u, 0, sm);
    uint32_t nkey;     // smallest probability bits in the nucleus
    int64_t nlim;      // entries of bits nkey with index < nlim belong to it
    long long last;    // the nucleus' last entry in sorted order (the reference's pi[n-1])
    double cum;        // the nucleus mass (the reference's cum)
    if (sm.found) {
        nkey = sm.key;
        const float pk = __uint_as_float(nkey);
        if (threadIdx.x == 0) {  // tied entries of probability pk, in index order, until the mass reaches top_p
            double c = (double)sm.above / SP_FIX;
            unsigned j = 0;
            do { c += (double)pk; j++; } while (c < tp && j < sm.ties);
            sm.dscr[0] = c;
            sm.iscr[0] = (int)j;
        }
        __syncthreads();
        cum = sm.dscr[0];
        const int j = sm.iscr[0];
        __syncthreads();
        last = sp_nth_equal(pr, V, nkey, V, j - 1, sm);
        nlim = last + 1;
    } else {  // the row's whole mass stays below top_p: every entry
        nkey = 0u;
        nlim = V;
        double tot = 0.0;
        uint32_t kmin = 0xffffffffu;
        for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
            tot += (double)pr[i];
            kmin = min(kmin, __float_as_uint(pr[i]));
        }
        cum = sp_reduce(tot, sm.dscr, [](double a, double b) { return a + b; });
        kmin = sp_reduce(kmin, (uint32_t *)sm.iscr, [](uint32_t a, uint32_t b) { return a < b ? a : b; });
        // last in sorted order: the smallest probability, highest index among equals
        long long li = -1;
        for (int64_t i = threadIdx.x; i < V; i += blockDim.x)
            if (__float_as_uint(pr[i]) == kmin) li = i;
        last = sp_reduce(li, sm.lscr, [](long long a, long long b) { return a > b ? a : b; });
    }
    // r and the walk along the nucleus
    uint64_t st = rng[row];
    const float r = sp_rng_f(st) * (float)cum;
    const unsigned long long rfix = (unsigned long long)((double)r * SP_FIX);
    long long pick = -1;
    sp_search(pr, V, rfix ? rfix : 1ull, nkey, nlim, sm);  // r == 0 stops at the first entry
    if (sm.found) {
        const uint32_t key = sm.key;
        const unsigned long long pkf = sp_fix(__uint_as_float(key));
        const unsigned long long need = (rfix ? rfix : 1ull) - sm.above;
        long long t = pkf ? (long long)((need + pkf - 1) / pkf) - 1 : 0;
        if (t < 0) t = 0;
        pick = sp_nth_equal(pr, V, key, key == nkey ? nlim : V, t, sm);
    }
    if (threadIdx.x == 0) {
        rng[row] = st;
        out[row] = (int32_t)(pick >= 0 ? pick : last);
    }
}

size_t sample_smem_bytes() { return sizeof(SpSmem); }

int sample_topp(const float *logits, int64_t ldl, int64_t V, int n_rows, float temp, float topp, uint64_t *rng,
                int32_t *out, float *probs, cudaStream_t st) {
    MG_REQUIRE(logits && out && V > 0 && n_rows >= 0 && ldl >= V, MG_ERR_ARG, "sample: bad arguments");
    MG_REQUIRE(temp <= 0.f || (rng && probs), MG_ERR_ARG, "sample: temperature > 0 needs rng states and scratch");
    MG_REQUIRE(V < (1LL << 31), MG_ERR_ARG, "sample: vocabulary too large");
    if (n_rows == 0) return MG_OK;
    const size_t smem = sizeof(SpSmem);
    k_sample_topp<<<n_rows, SP_THREADS, smem, st>>>(logits, ldl, V, temp, topp, rng, out, probs);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

}  // namespace mg
