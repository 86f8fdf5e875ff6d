// Device generator for the seeded synthetic workload; produces the same bytes as
// stratacuda_b200/synth.py (counter-based SplitMix64, Box-Muller with a log/cos built from
// correctly rounded +, -, *, / and sqrt only, every step rounded separately).
#include "common.cuh"
#include "kernels.h"

namespace strata {
namespace {

constexpr unsigned long long kGamma = 0x9E3779B97F4A7C15ull;
constexpr unsigned long long kSub = 0xD1B54A32D192ED03ull;
constexpr double kLn2 = 0.6931471805599453;
constexpr double kTwoPi = 6.283185307179586;

__host__ __device__ inline unsigned long long mix(unsigned long long z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ inline unsigned long long draw(unsigned long long key, unsigned long long i) { return mix(key + (i + 1) * kGamma); }
__device__ inline double uniform(unsigned long long r) { return __dmul_rn(__dadd_rn((double)(r >> 11), 0.5), 0x1p-53); }

__device__ double det_log(double u) {
    unsigned long long bits = (unsigned long long)__double_as_longlong(u);
    long long e = (long long)((bits >> 52) & 0x7FFull) - 1023;
    double m = __longlong_as_double((long long)((bits & 0x000FFFFFFFFFFFFFull) | 0x3FF0000000000000ull));
    if (m > 1.4142135623730951) {
        m = __dmul_rn(m, 0.5);
        e += 1;
    }
    double s = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0));
    double s2 = __dmul_rn(s, s);
    double term = s, acc = s;
    for (int n = 3; n < 22; n += 2) {
        term = __dmul_rn(term, s2);
        acc = __dadd_rn(acc, __ddiv_rn(term, (double)n));
    }
    return __dadd_rn(__dmul_rn((double)e, kLn2), __dmul_rn(2.0, acc));
}

__device__ double det_cos_turns(double v) {
    double w = v > 0.5 ? __dsub_rn(v, 1.0) : v;
    w = fabs(w);
    bool flip = w > 0.25;
    if (flip) w = __dsub_rn(0.5, w);
    double a = __dmul_rn(w, kTwoPi);
    double a2 = __dmul_rn(a, a);
    double term = 1.0, acc = 1.0;
    for (int n = 2; n < 24; n += 2) {
        term = __ddiv_rn(__dmul_rn(term, a2), (double)(-(n - 1) * n));
        acc = __dadd_rn(acc, term);
    }
    return flip ? -acc : acc;
}

__device__ double normal_at(unsigned long long key, unsigned long long n) {
    double u1 = uniform(draw(key, 2 * n)), u2 = uniform(draw(key, 2 * n + 1));
    return __dmul_rn(__dsqrt_rn(__dmul_rn(-2.0, det_log(u1))), det_cos_turns(u2));
}

__host__ __device__ inline unsigned long long key_of(unsigned long long seed, unsigned long long tag, unsigned long long sub) {
    return mix(mix(seed + tag * kGamma) + sub * kSub);
}

// flags: 1 = the shared expert's streams, 2 = signed scales N(0, 0.02) instead of |N(0, 0.02)|
__global__ void k_blobs(unsigned *out, unsigned long long seed, int layer, int first, int count, long long code_words, long long words,
                        int flags) {
    const bool shared = flags & 1, sign = flags & 2;
    long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)count * words) return;
    int e = first + (int)(idx / words);
    long long w = idx % words;
    unsigned long long sub = ((unsigned long long)layer << 20) | (unsigned long long)e;
    if (w < code_words) {
        out[idx] = (unsigned)(draw(key_of(seed, shared ? 6 : 3, sub), (unsigned long long)w) & 0xFFFFFFFFull);
    } else {
        unsigned long long hp = (unsigned long long)(w - code_words), sk = key_of(seed, shared ? 7 : 4, sub);
        const double z0 = __dmul_rn(normal_at(sk, 2 * hp), 0.02), z1 = __dmul_rn(normal_at(sk, 2 * hp + 1), 0.02);
        __half h0 = __double2half(sign ? z0 : fabs(z0));
        __half h1 = __double2half(sign ? z1 : fabs(z1));
        out[idx] = (unsigned)__half_as_ushort(h0) | ((unsigned)__half_as_ushort(h1) << 16);
    }
}

__global__ void k_normals(float *out, unsigned long long key, long long start, long long count, double scale) {
    long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= count) return;
    double z = normal_at(key, (unsigned long long)(start + n));
    out[n] = __double2float_rn(__dmul_rn(z, scale));
}

}  // namespace

unsigned long long synth_stream_key(unsigned long long seed, unsigned long long tag, unsigned long long sub) {
    return key_of(seed, tag, sub);
}

cudaError_t synth_expert_blobs(unsigned *out, unsigned long long seed, int layer, int first_expert, int count, int width, int ff,
                               int shared, cudaStream_t s) {
    long long code_words = 3LL * ff * width / 16, words = code_words + 3LL * ff * width / 128;
    long long n = (long long)count * words;
    k_blobs<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(out, seed, layer, first_expert, count, code_words, words, shared);
    return cudaGetLastError();
}

cudaError_t synth_normals_f32(float *out, unsigned long long key, long long start, long long count, double scale, cudaStream_t s) {
    k_normals<<<(unsigned)((count + 255) / 256), 256, 0, s>>>(out, key, start, count, scale);
    return cudaGetLastError();
}

}  // namespace strata
