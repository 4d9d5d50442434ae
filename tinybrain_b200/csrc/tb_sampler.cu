// tb_sampler.cu -- device sampler after the LM head (Sampler.swift:401-473,
// Sampler.sampleDetailed; step bookkeeping as ModelRunner.swift:251-292).
//
// One 1024-thread CTA per sequence keeps the sequence's logits row in shared
// memory (a global working row when the vocabulary is too large) and runs the
// reference's five steps on it:
//   1. repetition penalty, sign-aware, applied once per history entry
//      (prompt + generated tokens).  Every entry applies the same map
//      f(x) = x > 0 ? x / pen : x * pen, so the entries of one token are
//      applied in any order with an atomic compare-and-swap and the result is
//      exactly f^count(x);
//   2. top-k, else top-p: the reference sorts (descending value; equal
//      values here keep ascending index) and keeps a prefix.  The prefix
//      boundary is found without sorting, by a radix select over the
//      order-preserving 32-bit key of the value (8-bit digits, four passes,
//      per-warp histograms): top-k counts elements, top-p accumulates their
//      softmax mass (in fp64) until it reaches top_p.  Ties at the boundary
//      key are resolved by a second select over the indices;
//   3. temperature (below 0.01 the logits stay unscaled);
//   4. softmax with the reference's +1e-7 denominator, entropy -sum p log p;
//   5. the LCG draw (Sampler.swift:369-381) and the first index whose
//      running CDF reaches the threshold (Sampler.swift:340-359), scanned in
//      index order 1024 elements at a time.
// Sums are parallel reductions, so the running sums differ from the
// reference's sequential float sums in the last bits: a draw whose threshold
// lies within rounding of a CDF boundary (or a top-p mass within rounding of
// top_p) may pick the neighbouring element.
#include <cfloat>

#include "tb_common.cuh"
#include "tb_unit.cuh"

namespace tb {
namespace {

constexpr int kSampThreads = 1024;
constexpr int kSampWarps = kSampThreads / 32;
constexpr int kBins = 256;
// shared layout: per-warp histograms | bin totals | reduction scratch | row
constexpr size_t kHistBytes = (size_t)kSampWarps * kBins * sizeof(double);
constexpr size_t kTotBytes = kBins * sizeof(double);
constexpr size_t kRedBytes = 128 * sizeof(double);
constexpr size_t kSampHead = kHistBytes + kTotBytes + kRedBytes;
constexpr size_t kSampSmemMax = 227 * 1024;

struct Shared {
    double* hist;  // [warps][bins]
    double* tot;   // [bins]
    double* red;   // scratch: reductions, select results
};

__device__ __forceinline__ float block_max(float v, double* red) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    float* r = reinterpret_cast<float*>(red);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = r[0];
    for (int w = 1; w < kSampWarps; ++w) m = fmaxf(m, r[w]);
    return m;
}

// Fixed-order block sum (the same result on every thread and every run).
__device__ __forceinline__ float block_sum(float v, double* red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    float* r = reinterpret_cast<float*>(red);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.0f;
    for (int w = 0; w < kSampWarps; ++w) s += r[w];
    return s;
}

__device__ __forceinline__ double block_sum_d(double v, double* red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    double s = 0.0;
    for (int w = 0; w < kSampWarps; ++w) s += red[w];
    return s;
}

// Radix select over the descending order of (key, then index ascending) of
// the members: the key T of the element at which the running weight first
// reaches `target`.  Returns false when the members' total weight stays below
// target.  *above = weight of the members with key > T, *at = weight of
// those with key == T.
template <class Member, class Key, class Weight>
__device__ bool radix_select(int n, Member member, Key key, Weight weight, double target, const Shared& sh,
                             uint32_t* T, double* above, double* at) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t prefix = 0, pmask = 0;
    double acc_above = 0.0, at_w = 0.0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < kSampWarps * kBins; i += kSampThreads) sh.hist[i] = 0.0;
        __syncthreads();
        double* hw = sh.hist + warp * kBins;
        for (int i = tid; i < n; i += kSampThreads) {
            if (!member(i)) continue;
            const uint32_t k = key(i);
            if ((k & pmask) != prefix) continue;
            const double w = weight(i);
            if (w != 0.0) atomicAdd(hw + ((k >> shift) & 0xFF), w);
        }
        __syncthreads();
        if (tid < kBins) {
            double s = 0.0;
            for (int w = 0; w < kSampWarps; ++w) s += sh.hist[w * kBins + tid];
            sh.tot[tid] = s;
        }
        __syncthreads();
        if (warp == 0) {
            // lane l owns bins 8l..8l+7; weight of the bins above lane l's
            double s = 0.0;
            for (int j = 0; j < 8; ++j) s += sh.tot[lane * 8 + j];
            double incl = s;  // suffix sum over lanes >= l
            for (int o = 1; o < 32; o <<= 1) {
                const double t = __shfl_down_sync(0xffffffffu, incl, o);
                if (lane + o < 32) incl += t;
            }
            double acc = acc_above + (incl - s);
            int found = -1;
            double f_above = 0.0;
            for (int j = 7; j >= 0; --j) {
                const double t = sh.tot[lane * 8 + j];
                if (found < 0 && t != 0.0 && acc + t >= target) {
                    found = lane * 8 + j;
                    f_above = acc;
                }
                acc += t;
            }
            const unsigned ok = __ballot_sync(0xffffffffu, found >= 0);
            if (ok) {
                const int src = 31 - __clz(ok);  // the highest bin that reaches target
                if (lane == src) {
                    sh.red[64] = f_above;
                    sh.red[65] = sh.tot[found];
                    sh.red[66] = (double)found;
                }
            } else if (lane == 0) {
                sh.red[66] = -1.0;
            }
        }
        __syncthreads();
        const int bin = (int)sh.red[66];
        if (bin < 0) {
            __syncthreads();
            return false;
        }
        acc_above = sh.red[64];
        at_w = sh.red[65];
        prefix |= (uint32_t)bin << shift;
        pmask |= 0xFFu << shift;
        __syncthreads();
    }
    *T = prefix;
    *above = acc_above;
    *at = at_w;
    return true;
}

__global__ void __launch_bounds__(kSampThreads, 1) sample_kernel(SampleParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    Shared sh;
    sh.hist = reinterpret_cast<double*>(smem);
    sh.tot = reinterpret_cast<double*>(smem + kHistBytes);
    sh.red = reinterpret_cast<double*>(smem + kHistBytes + kTotBytes);
    const int m = blockIdx.x, tid = threadIdx.x, V = p.V;
    float* x = p.work ? p.work + (size_t)m * V : reinterpret_cast<float*>(smem + kSampHead);

    pdl_wait();
    pdl_launch_dependents();
    SeqState& sq = p.seq[m];
    const int active = sq.active, pos = sq.pos, n_prompt = sq.n_prompt, n_out = sq.n_out, max_out = sq.max_out;
    if (!active || pos < n_prompt - 1) {
        if (active && (p.logprob_acc || p.logprob_out)) {
            // PerplexityHarness.computePerplexity (PerplexityHarness.swift:155-186):
            // log P(target) = logit[target] - (log(sum exp(logit - max)) + max),
            // the max in fp32, the exponentials and their sum in fp64
            const float* lg = p.logits + (size_t)m * V;
            float lm = -INFINITY;
            for (int i = tid; i < V; i += kSampThreads) lm = fmaxf(lm, lg[i]);
            const float mx = block_max(lm, sh.red);
            double ls = 0.0;
            for (int i = tid; i < V; i += kSampThreads) ls += exp((double)lg[i] - (double)mx);
            const double tot = block_sum_d(ls, sh.red);
            if (tid == 0) {
                const int tgt = p.target ? p.target[m] : p.prompt[(size_t)m * p.prompt_stride + pos + 1];
                const double lp = (double)lg[tgt] - (log(tot) + (double)mx);
                if (p.logprob_out)
                    p.logprob_out[m] = lp;
                else
                    p.logprob_acc[m] += lp;
            }
        }
        __syncthreads();
        if (tid == 0) {
            if (active) {  // prompt step: feed the next prompt token
                sq.token = p.target ? p.target[m] : p.prompt[(size_t)m * p.prompt_stride + pos + 1];
                sq.pos = pos + 1;
            }
            sq.best = 0ull;
            if (m == 0 && p.ar_step) *p.ar_step += 1u;
        }
        return;
    }

    const float* lg = p.logits + (size_t)m * V;
    for (int i = tid; i < V; i += kSampThreads) x[i] = lg[i];
    __syncthreads();

    // 1. repetition penalty over prompt + generated tokens
    const float pen = p.repetition_penalty;
    const int n_gen = n_out < max_out ? n_out : max_out;
    const int n_hist = n_prompt + n_gen;
    if (pen != 1.0f && n_hist > 0) {
        for (int h = tid; h < n_hist; h += kSampThreads) {
            const int t = h < n_prompt ? p.prompt[(size_t)m * p.prompt_stride + h]
                                       : p.out_tokens[(size_t)m * max_out + (h - n_prompt)];
            if (t < 0 || t >= V) continue;
            unsigned int* a = reinterpret_cast<unsigned int*>(x + t);
            unsigned int old = *a, assumed;
            do {
                assumed = old;
                const float v = __uint_as_float(assumed);
                const float nv = v > 0.0f ? __fdiv_rn(v, pen) : __fmul_rn(v, pen);
                old = atomicCAS(a, assumed, __float_as_uint(nv));
            } while (old != assumed);
        }
        __syncthreads();
    }

    // 2. top-k, else top-p
    const bool do_k = p.top_k > 0 && p.top_k < V;
    const bool do_p = p.top_k <= 0 && p.has_top_p;
    if (do_k || do_p) {
        float mx = 0.0f, den = 0.0f;
        if (do_p) {
            float lm = -INFINITY;
            for (int i = tid; i < V; i += kSampThreads) lm = fmaxf(lm, x[i]);
            mx = block_max(lm, sh.red);
            float ls = 0.0f;
            for (int i = tid; i < V; i += kSampThreads) ls += expf(x[i] - mx);
            den = block_sum(ls, sh.red) + 1e-7f;  // softmax denominator (Tensor softmax)
        }
        auto prob = [&](int i) { return __fdiv_rn(expf(x[i] - mx), den); };
        auto all = [](int) { return true; };
        auto vkey = [&](int i) { return float_order_key(do_k ? x[i] : prob(i)); };
        uint32_t T = 0;
        double above = 0.0, at = 0.0;
        bool reached;
        if (do_k) {
            reached = radix_select(V, all, vkey, [](int) { return 1.0; }, (double)p.top_k, sh, &T, &above, &at);
        } else {
            const double target = fmax((double)p.top_p, 1e-300);
            reached = radix_select(V, all, vkey, [&](int i) { return (double)prob(i); }, target, sh, &T, &above,
                                   &at);
        }
        if (reached) {
            // how many elements of the boundary key the prefix takes
            long long eq_n, need;
            if (do_k) {
                eq_n = llround(at);
                need = (long long)p.top_k - llround(above);
            } else {
                const double v = (double)float_from_order_key(T);
                eq_n = v > 0.0 ? llround(at / v) : 1;
                need = v > 0.0 ? (long long)ceil(((double)p.top_p - above) / v) : eq_n;
            }
            need = need < 1 ? 1 : need;
            uint32_t last_idx_key = 0;  // keep boundary-key elements with index <= ~last_idx_key
            bool all_ties = need >= eq_n;
            if (!all_ties) {
                double a2 = 0.0, t2 = 0.0;
                radix_select(V, [&](int i) { return vkey(i) == T; }, [](int i) { return ~(uint32_t)i; },
                             [](int) { return 1.0; }, (double)need, sh, &last_idx_key, &a2, &t2);
            }
            const uint32_t max_idx = ~last_idx_key;
            // each element's key depends on its own value only, so it is masked in place
            for (int i = tid; i < V; i += kSampThreads) {
                const uint32_t k = vkey(i);
                const bool keep = k > T || (k == T && (all_ties || (uint32_t)i <= max_idx));
                if (!keep) x[i] = -INFINITY;
            }
            __syncthreads();
        }
    }

    // 3. temperature; 4. final softmax and entropy
    const float temp = p.temperature > 0.0f ? p.temperature : 0.0f;
    const bool scale = !(temp < 0.01f);
    float lm = -INFINITY;
    for (int i = tid; i < V; i += kSampThreads) {
        float v = x[i];
        if (scale) {
            v = __fdiv_rn(v, temp);
            x[i] = v;
        }
        lm = fmaxf(lm, v);
    }
    const float mx = block_max(lm, sh.red);
    float ls = 0.0f;
    for (int i = tid; i < V; i += kSampThreads) {
        const float e = expf(x[i] - mx);
        x[i] = e;
        ls += e;
    }
    const float den = block_sum(ls, sh.red) + 1e-7f;
    float le = 0.0f;
    for (int i = tid; i < V; i += kSampThreads) {
        const float q = __fdiv_rn(x[i], den);
        x[i] = q;
        if (q > 0.0f) le -= q * logf(q);
    }
    const float entropy = block_sum(le, sh.red);

    // 5. LCG draw and CDF scan in index order
    unsigned long long st = p.rng[m];
    st = st * 6364136223846793005ull + 1442695040888963407ull;
    const float threshold = __fdiv_rn(__ull2float_rn(st), 18446744073709551616.0f);  // Float(UInt64.max) = 2^64
    float* wsum = reinterpret_cast<float*>(sh.red);  // [0, 32) warp sums, [32] tile total
    int* found = reinterpret_cast<int*>(sh.red + 40);
    if (tid == 0) *found = V - 1;  // the reference's fallback
    float carry = 0.0f;
    const int warp = tid >> 5, lane = tid & 31;
    for (int base = 0; base < V; base += kSampThreads) {
        const int i = base + tid;
        float v = i < V ? x[i] : 0.0f;
        for (int o = 1; o < 32; o <<= 1) {
            const float t = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += t;
        }
        __syncthreads();
        if (lane == 31) wsum[warp] = v;
        __syncthreads();
        if (warp == 0) {
            float w = wsum[lane];
            for (int o = 1; o < 32; o <<= 1) {
                const float t = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += t;
            }
            wsum[lane] = w;  // inclusive over warps
            if (lane == 31) wsum[32] = w;
        }
        __syncthreads();
        const float wex = warp ? wsum[warp - 1] : 0.0f;
        const float cum = carry + (wex + v);
        const bool hit = i < V && threshold <= cum;
        if (hit) atomicMin(found, i);
        const float tile = wsum[32];
        if (__syncthreads_or(hit)) break;
        carry += tile;
    }
    __syncthreads();
    if (tid == 0) {
        const int tok = *found;
        const float q = x[tok];
        if (n_out < max_out) {
            const size_t o = (size_t)m * max_out + n_out;
            p.out_tokens[o] = tok;
            if (p.out_prob) p.out_prob[o] = q;
            if (p.out_entropy) p.out_entropy[o] = entropy;
        }
        sq.n_out = n_out + 1;
        sq.token = tok;
        sq.pos = pos + 1;
        sq.best = 0ull;
        p.rng[m] = st;
        if (m == 0 && p.ar_step) *p.ar_step += 1u;
    }
}

}  // namespace

size_t sample_smem_bytes(int V, bool* in_smem) {
    const size_t full = kSampHead + (size_t)V * sizeof(float);
    const bool fits = full <= kSampSmemMax;
    if (in_smem) *in_smem = fits;
    return fits ? full : kSampHead;
}

cudaError_t launch_sample(const SampleParams& p, cudaStream_t stream, bool pdl) {
    bool in_smem = false;
    const size_t smem = sample_smem_bytes(p.V, &in_smem);
    if (!in_smem && !p.work) return cudaErrorInvalidValue;
    SampleParams q = p;
    if (in_smem) q.work = nullptr;
    cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)p.M);
    cfg.blockDim = dim3(kSampThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, sample_kernel, q);
}

}  // namespace tb
