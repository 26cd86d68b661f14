// CPU oracle for the SDPA hot path -- TEST INFRASTRUCTURE ONLY.
//
// This file restates, in plain C++, what the reference (SkillfulElectro/GGUF_train) computes on
// the scaled-dot-product-attention path, so that the CUDA kernels can be checked against it.
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it, and only as the
// checker / the timed CPU baseline. The product library never links or calls it.
//
// Parity status: the reference's native library cannot be built here as a whole
// (csrc/gt_internal.h:4-8 needs ggml headers that build_native.py:217-307 downloads), but its SDPA
// forward, gt_flash_attention (csrc/gt_ops_nn.cpp:2423-2525), uses none of ggml: oracle/build_ref.py
// compiles that function from the reference source into oracle/_ref/, and the forward below is
// pinned to it (bit for bit for f32/f16/bf16 outputs, masks and causal included; tests/
// test_oracle_ref.py and the fixture tests/golden/ref_flash_attention.npz). The backward (a chain of
// ggml ops in the reference) and the Q8_0 codec are pinned against independent implementations
// (torch float64 SDPA and autograd; gguf-py's Q8_0, which states bit-exactness with ggml-quants.c).
//
// Every routine cites the reference lines it follows. Nothing here is copied from the reference;
// the loops are written from the behaviour those lines define.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <mutex>
#include <random>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// gt_dtype codes, gguf_train.h:22-36
enum { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2, DT_F64 = 3, DT_BOOL = 9 };

std::mutex g_rng_mtx;
std::mt19937_64 g_rng;  // one global engine, as gt_runtime_state::rng (gt_core.cpp:136-141)

uint32_t f32_bits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
float bits_f32(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// IEEE binary32 -> binary16, round to nearest even, subnormals kept, overflow -> inf.
// Restated from the IEEE 754 definition (ggml_fp32_to_fp16, gt_internal.h:265).
uint16_t f32_to_f16(float f) {
    uint32_t x = f32_bits(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);          // NaN
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);         // rounds to >= 65520 -> inf
    if (ax < 0x38800000u) {                                            // below 2^-14: subnormal half
        // value = ax as float; half subnormal unit is 2^-24
        float a = bits_f32(ax);
        // a * 2^24 rounded to nearest even integer (exact in double)
        double s = (double)a * 16777216.0;
        double r = std::nearbyint(s);  // default rounding mode: nearest even
        return (uint16_t)(sign | (uint32_t)r);
    }
    uint32_t e = (ax >> 23) - 127 + 15;
    uint32_t m = ax & 0x7fffffu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;         // carry may bump exponent: fine
    return (uint16_t)(sign | h);
}

float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    if (e == 0) {
        float v = (float)m * (1.0f / 16777216.0f);
        return sign ? -v : v;
    }
    if (e == 31) return bits_f32(sign | 0x7f800000u | (m << 13));
    return bits_f32(sign | ((e - 15 + 127) << 23) | (m << 13));
}

// binary32 -> bfloat16, round to nearest even, NaN kept quiet (ggml_fp32_to_bf16, gt_internal.h:266)
uint16_t f32_to_bf16(float f) {
    uint32_t u = f32_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

float bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

// The value a double takes after gt_write_f64_at(dtype) and gt_read_f64_at(dtype)
// (gt_internal.h:243-277): through float, then to the storage type.
double round_to_dtype(double v, int dtype) {
    switch (dtype) {
        case DT_F64: return v;
        case DT_F32: return (double)(float)v;
        case DT_F16: return (double)f16_to_f32(f32_to_f16((float)v));
        case DT_BF16: return (double)bf16_to_f32(f32_to_bf16((float)v));
        case DT_BOOL: return v != 0.0 ? 1.0 : 0.0;
        default: return v;
    }
}

int set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
    return omp_get_max_threads();
#else
    (void)nthreads;
    return 1;
#endif
}

// Mask element index for (b, h, l, s), following the broadcast rules of gt_ops_nn.cpp:2489-2494:
// a 2-D mask (L|1, S|1) or a 4-D mask (B|1, H|1, L|1, S|1), size-1 dims broadcast.
inline int64_t mask_index(int mask_ndim, const int64_t* ms, int64_t b, int64_t h, int64_t l, int64_t s) {
    if (mask_ndim == 2) return (ms[0] > 1 ? l : 0) * ms[1] + (ms[1] > 1 ? s : 0);
    int64_t mb = ms[0] > 1 ? b : 0;
    int64_t mh = ms[1] > 1 ? h : 0;
    return ((mb * ms[1] + mh) * ms[2] + (ms[2] > 1 ? l : 0)) * ms[3] + (ms[3] > 1 ? s : 0);
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- seeded inputs (gt_core.cpp)

// gt_manual_seed, gt_core.cpp:136-141: reseed the single global mt19937_64.
void orc_manual_seed(uint64_t seed) {
    std::lock_guard<std::mutex> lk(g_rng_mtx);
    g_rng.seed(seed);
}

// gt_fill_normal, gt_core.cpp:1199-1215: a fresh normal_distribution<double>(mean, std) per call,
// values drawn in row-major order. std == 0 writes the mean without drawing.
int orc_fill_normal(double* out, int64_t n, double mean, double stdv) {
    std::lock_guard<std::mutex> lk(g_rng_mtx);
    std::normal_distribution<double> dist(mean, stdv > 0.0 ? stdv : 1e-30);
    for (int64_t i = 0; i < n; ++i) out[i] = (stdv == 0.0) ? mean : dist(g_rng);
    return 0;
}

// Raw 64-bit outputs of the engine after seeding (for the C++ standard's known-answer check of
// mt19937_64: the 10000th output of a default-seeded engine is 9981545732273789042).
void orc_engine_raw(uint64_t seed, int64_t n, uint64_t* out) {
    std::lock_guard<std::mutex> lk(g_rng_mtx);
    std::mt19937_64 e(seed);
    for (int64_t i = 0; i < n; ++i) out[i] = e();
}

// gt_fill_uniform, gt_core.cpp:1182-1197
int orc_fill_uniform(double* out, int64_t n, double lo, double hi) {
    std::lock_guard<std::mutex> lk(g_rng_mtx);
    std::uniform_real_distribution<double> dist(lo, hi);
    for (int64_t i = 0; i < n; ++i) out[i] = dist(g_rng);
    return 0;
}

// gt_fill_bernoulli_prob, gt_core.cpp:1283-1298
int orc_fill_bernoulli(double* out, int64_t n, double p) {
    std::lock_guard<std::mutex> lk(g_rng_mtx);
    std::bernoulli_distribution dist(std::min(1.0, std::max(0.0, p)));
    for (int64_t i = 0; i < n; ++i) out[i] = dist(g_rng) ? 1.0 : 0.0;
    return 0;
}

// ---------------------------------------------------------------- dtype storage semantics

void orc_round_to_dtype(const double* in, int64_t n, int dtype, double* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = round_to_dtype(in[i], dtype);
}

// Store values as the dtype's bits (f32: 4 B, f16/bf16: 2 B, f64: 8 B, bool: 1 B).
int orc_to_bits(const double* in, int64_t n, int dtype, void* out) {
    for (int64_t i = 0; i < n; ++i) {
        switch (dtype) {
            case DT_F32: ((float*)out)[i] = (float)in[i]; break;
            case DT_F64: ((double*)out)[i] = in[i]; break;
            case DT_F16: ((uint16_t*)out)[i] = f32_to_f16((float)in[i]); break;
            case DT_BF16: ((uint16_t*)out)[i] = f32_to_bf16((float)in[i]); break;
            case DT_BOOL: ((uint8_t*)out)[i] = in[i] != 0.0; break;
            default: return -1;
        }
    }
    return 0;
}

int orc_from_bits(const void* in, int64_t n, int dtype, double* out) {
    for (int64_t i = 0; i < n; ++i) {
        switch (dtype) {
            case DT_F32: out[i] = ((const float*)in)[i]; break;
            case DT_F64: out[i] = ((const double*)in)[i]; break;
            case DT_F16: out[i] = f16_to_f32(((const uint16_t*)in)[i]); break;
            case DT_BF16: out[i] = bf16_to_f32(((const uint16_t*)in)[i]); break;
            case DT_BOOL: out[i] = ((const uint8_t*)in)[i] ? 1.0 : 0.0; break;
            default: return -1;
        }
    }
    return 0;
}

// ---------------------------------------------------------------- forward

// Restatement of gt_flash_attention, csrc/gt_ops_nn.cpp:2423-2525.
//   q (B,H,L,D), k (B,Hkv,S,D), v (B,Hkv,S,Dv), contiguous, values already in double.
//   mask: nullptr, or a contiguous 2-D / 4-D array with broadcast dims (mask_is_bool: 0/1 values,
//   0 = may not attend; else additive).
//   Per (b, h) and query row l (:2468-2522): scores in double, dot *= (double)scale, causal s > l
//   (top-left) -> -inf, bool false -> -inf, float mask added; max; exp(x - max) and sum over the
//   finite scores; inv = sum > 0 ? 1/sum : 0 (a row with no finite score gives 0); out =
//   sum_s p * v with p == 0 skipped. The caller stores out through float into q's dtype.
//   GQA maps query head h to kv head h / (H / Hkv) (:2471). scale <= 0 -> 1/sqrt(D) (:2433).
int orc_sdpa_fwd(const double* q, const double* k, const double* v,
                 int64_t B, int64_t H, int64_t Hkv, int64_t L, int64_t S, int64_t D, int64_t Dv,
                 const double* mask, int mask_ndim, const int64_t* mask_shape, int mask_is_bool,
                 float scale, int is_causal, double* out, int nthreads) {
    if (Hkv <= 0 || H % Hkv != 0) return -1;
    const int64_t group = H / Hkv;
    if (scale <= 0.0f) scale = 1.0f / std::sqrt((float)D);
    set_threads(nthreads);
    const double ninf = -std::numeric_limits<double>::infinity();

#pragma omp parallel for collapse(2) schedule(dynamic, 1) if (B * H > 4)
    for (int64_t b = 0; b < B; ++b) {
        for (int64_t h = 0; h < H; ++h) {
            const int64_t hk = h / group;
            std::vector<double> sc(S);
            const double* kb = k + (b * Hkv + hk) * S * D;
            const double* vb = v + (b * Hkv + hk) * S * Dv;
            for (int64_t l = 0; l < L; ++l) {
                const double* qr = q + ((b * H + h) * L + l) * D;
                double mx = ninf;
                for (int64_t s = 0; s < S; ++s) {
                    if (is_causal && s > l) { sc[s] = ninf; continue; }
                    double dot = 0.0;
                    const double* kr = kb + s * D;
                    for (int64_t d = 0; d < D; ++d) dot += qr[d] * kr[d];
                    dot *= (double)scale;
                    if (mask) {
                        double mv = mask[mask_index(mask_ndim, mask_shape, b, h, l, s)];
                        if (mask_is_bool) { if (mv == 0.0) dot = ninf; }
                        else dot += mv;
                    }
                    sc[s] = dot;
                    if (dot > mx) mx = dot;
                }
                double se = 0.0;
                for (int64_t s = 0; s < S; ++s) {
                    if (std::isinf(sc[s]) && sc[s] < 0) sc[s] = 0.0;
                    else { sc[s] = std::exp(sc[s] - mx); se += sc[s]; }
                }
                const double inv = se > 0.0 ? 1.0 / se : 0.0;
                double* orow = out + ((b * H + h) * L + l) * Dv;
                // the reference loops dv outer, s inner (:2511-2519); the sum order per output
                // element is the same (s ascending), so this loop order gives identical doubles
                for (int64_t dv = 0; dv < Dv; ++dv) orow[dv] = 0.0;
                for (int64_t s = 0; s < S; ++s) {
                    const double p = sc[s] * inv;
                    if (p == 0.0) continue;
                    const double* vr = vb + s * Dv;
                    for (int64_t dv = 0; dv < Dv; ++dv) orow[dv] += p * vr[dv];
                }
            }
        }
    }
    return 0;
}

// Same as orc_sdpa_fwd but with the reference's literal loop order and V access pattern
// (dv outer, s inner, V read with stride Dv: gt_ops_nn.cpp:2511-2519). Used only as the timed
// CPU baseline so that its memory behaviour matches the reference's loop. q holds query rows
// q_offset .. q_offset+L-1 of a longer sequence (causal masking uses the absolute row index), so a
// bounded slice of a large workload can be timed with its exact amount of work.
int orc_sdpa_fwd_reforder(const double* q, const double* k, const double* v,
                          int64_t B, int64_t H, int64_t Hkv, int64_t L, int64_t S, int64_t D, int64_t Dv,
                          float scale, int is_causal, int64_t q_offset, double* out, int nthreads) {
    if (Hkv <= 0 || H % Hkv != 0) return -1;
    const int64_t group = H / Hkv;
    if (scale <= 0.0f) scale = 1.0f / std::sqrt((float)D);
    set_threads(nthreads);
    const double ninf = -std::numeric_limits<double>::infinity();
#pragma omp parallel for collapse(2) if (B * H > 4)
    for (int64_t b = 0; b < B; ++b) {
        for (int64_t h = 0; h < H; ++h) {
            const int64_t hk = h / group;
            std::vector<double> sc(S);
            for (int64_t l = 0; l < L; ++l) {
                double mx = ninf;
                for (int64_t s = 0; s < S; ++s) {
                    if (is_causal && s > l + q_offset) { sc[s] = ninf; continue; }
                    double dot = 0.0;
                    const int64_t qo = ((b * H + h) * L + l) * D;
                    const int64_t ko = ((b * Hkv + hk) * S + s) * D;
                    for (int64_t d = 0; d < D; ++d) dot += q[qo + d] * k[ko + d];
                    dot *= (double)scale;
                    sc[s] = dot;
                    if (dot > mx) mx = dot;
                }
                double se = 0.0;
                for (int64_t s = 0; s < S; ++s) {
                    if (std::isinf(sc[s]) && sc[s] < 0) sc[s] = 0.0;
                    else { sc[s] = std::exp(sc[s] - mx); se += sc[s]; }
                }
                const double inv = se > 0.0 ? 1.0 / se : 0.0;
                const int64_t oo = ((b * H + h) * L + l) * Dv;
                for (int64_t dv = 0; dv < Dv; ++dv) {
                    double acc = 0.0;
                    for (int64_t s = 0; s < S; ++s) {
                        const double p = sc[s] * inv;
                        if (p == 0.0) continue;
                        acc += p * v[((b * Hkv + hk) * S + s) * Dv + dv];
                    }
                    out[oo + dv] = acc;
                }
            }
        }
    }
    return 0;
}

// ---------------------------------------------------------------- backward

// Restatement of FlashAttentionFn.backward, gguf_train/_functions.py:1934-1965, in double:
//   scores = q k^T * scale;  causal: + (-1e9) where s > l (added, :1944-1946);
//   bool mask: scores = -1e9 where mask is false (replaced, :1948-1949); float mask: added;
//   probs = softmax(scores, -1);  dv = probs^T dO;  dp = dO v^T;
//   ds = probs * (dp - sum(dp * probs, -1));  dq = ds k * scale;  dk = ds^T q * scale;
//   GQA: dk, dv summed over the H / Hkv query heads of each kv head (:1958-1962).
// Row blocks are streamed so no (L, S) buffer is held: memory per thread is rows_blk x S.
int orc_sdpa_bwd(const double* q, const double* k, const double* v, const double* dout,
                 int64_t B, int64_t H, int64_t Hkv, int64_t L, int64_t S, int64_t D, int64_t Dv,
                 const double* mask, int mask_ndim, const int64_t* mask_shape, int mask_is_bool,
                 double scale, int is_causal, double* dq, double* dk, double* dv, int nthreads) {
    if (Hkv <= 0 || H % Hkv != 0) return -1;
    const int64_t group = H / Hkv;
    const int threads = set_threads(nthreads);
    std::fill(dk, dk + B * Hkv * S * D, 0.0);
    std::fill(dv, dv + B * Hkv * S * Dv, 0.0);
    const int64_t RB = 64;
    const int64_t nblk = (L + RB - 1) / RB;
    // Tasks: (b, kv head, part), each part a share of the group's (query head, row block) pairs.
    // With fewer groups than threads a group is split into parts with private dk/dv sums, added up
    // after the loop; otherwise each group is one task writing its own dk/dv. dq rows are disjoint.
    const int64_t groups = B * Hkv;
    const int64_t parts = std::max<int64_t>(1, std::min<int64_t>(threads / std::max<int64_t>(groups, 1), group * nblk));
    std::vector<double> priv(parts > 1 ? (size_t)(groups * parts * S * (D + Dv)) : 0);
    // Without a mask, a causally masked score (s > l) gets -1e9 and its probability exp(-1e9 - max)
    // is exactly 0 in double, since key 0 is always allowed and keeps the row maximum finite: those
    // dot products are skipped. With a mask the full row is formed as the reference forms it.
    const bool skip_causal = is_causal && !mask;

#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t task = 0; task < groups * parts; ++task) {
        const int64_t gi = task / parts, part = task % parts;
        const int64_t b = gi / Hkv, hk = gi % Hkv;
        const double* kb = k + (b * Hkv + hk) * S * D;
        const double* vb = v + (b * Hkv + hk) * S * Dv;
        double* dkb = parts > 1 ? priv.data() + (size_t)task * S * (D + Dv) : dk + (b * Hkv + hk) * S * D;
        double* dvb = parts > 1 ? dkb + S * D : dv + (b * Hkv + hk) * S * Dv;
        std::vector<double> P(RB * S), DP(RB * S);
        for (int64_t w = part; w < group * nblk; w += parts) {
            const int64_t h = hk * group + w / nblk;
            const int64_t l0 = (w % nblk) * RB;
            const int64_t nr = std::min(RB, L - l0);
            for (int64_t r = 0; r < nr; ++r) {
                const int64_t l = l0 + r;
                const double* qr = q + ((b * H + h) * L + l) * D;
                const double* gr = dout + ((b * H + h) * L + l) * Dv;
                double* pr = P.data() + r * S;
                double* dpr = DP.data() + r * S;
                const int64_t s_end = skip_causal ? std::min(S, l + 1) : S;
                double mx = -std::numeric_limits<double>::infinity();
                for (int64_t s = 0; s < s_end; ++s) {
                    double dot = 0.0;
                    const double* kr = kb + s * D;
                    for (int64_t d = 0; d < D; ++d) dot += qr[d] * kr[d];
                    double x = dot * scale;
                    if (is_causal && s > l) x += -1e9;
                    if (mask) {
                        double mv = mask[mask_index(mask_ndim, mask_shape, b, h, l, s)];
                        if (mask_is_bool) { if (mv == 0.0) x = -1e9; }
                        else x += mv;
                    }
                    pr[s] = x;
                    if (x > mx) mx = x;
                }
                double se = 0.0;
                for (int64_t s = 0; s < s_end; ++s) { pr[s] = std::exp(pr[s] - mx); se += pr[s]; }
                for (int64_t s = 0; s < s_end; ++s) pr[s] /= se;
                for (int64_t s = s_end; s < S; ++s) pr[s] = 0.0;
                double rs = 0.0;
                for (int64_t s = 0; s < s_end; ++s) {
                    double dot = 0.0;
                    const double* vr = vb + s * Dv;
                    for (int64_t d = 0; d < Dv; ++d) dot += gr[d] * vr[d];
                    dpr[s] = dot;
                    rs += dot * pr[s];
                }
                for (int64_t s = s_end; s < S; ++s) dpr[s] = 0.0;
                double* dqr = dq + ((b * H + h) * L + l) * D;
                for (int64_t d = 0; d < D; ++d) dqr[d] = 0.0;
                for (int64_t s = 0; s < s_end; ++s) {
                    const double ds = pr[s] * (dpr[s] - rs);
                    dpr[s] = ds;
                    const double* kr = kb + s * D;
                    for (int64_t d = 0; d < D; ++d) dqr[d] += ds * kr[d];
                }
                for (int64_t d = 0; d < D; ++d) dqr[d] *= scale;
            }
            // dv += P^T dO, dk += dS^T q * scale for this row block
            for (int64_t s = 0; s < S; ++s) {
                double* dvr = dvb + s * Dv;
                double* dkr = dkb + s * D;
                for (int64_t r = 0; r < nr; ++r) {
                    const int64_t l = l0 + r;
                    const double p = P[r * S + s];
                    const double ds = DP[r * S + s] * scale;
                    const double* gr = dout + ((b * H + h) * L + l) * Dv;
                    const double* qr = q + ((b * H + h) * L + l) * D;
                    if (p != 0.0) for (int64_t d = 0; d < Dv; ++d) dvr[d] += p * gr[d];
                    if (ds != 0.0) for (int64_t d = 0; d < D; ++d) dkr[d] += ds * qr[d];
                }
            }
        }
    }
    if (parts > 1) {
#pragma omp parallel for
        for (int64_t gi = 0; gi < groups; ++gi) {
            double* dkg = dk + gi * S * D;
            double* dvg = dv + gi * S * Dv;
            for (int64_t part = 0; part < parts; ++part) {
                const double* src = priv.data() + (size_t)(gi * parts + part) * S * (D + Dv);
                for (int64_t i = 0; i < S * D; ++i) dkg[i] += src[i];
                for (int64_t i = 0; i < S * Dv; ++i) dvg[i] += src[S * D + i];
            }
        }
    }
    return 0;
}

// ---------------------------------------------------------------- Q8_0 (GGUF block format)

// Q8_0 block: fp16 scale d, then 32 int8 quants: 34 bytes per 32 values. Quantisation follows
// ggml's reference row quantiser that gt_tensor_to_dtype reaches through ggml_quantize_chunk
// (csrc/gt_core.cpp:832; ggml at llama.cpp b12283): amax = max |x|, d = amax / 127 (float),
// id = d != 0 ? 1/d : 0, q = round-half-away-from-zero(x * id), d stored as fp16 (RNE).
int orc_q8_0_quantize(const float* x, int64_t n, uint8_t* out) {
    if (n % 32 != 0) return -1;
    for (int64_t blk = 0; blk < n / 32; ++blk) {
        const float* xb = x + blk * 32;
        uint8_t* ob = out + blk * 34;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = std::max(amax, std::fabs(xb[j]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = f32_to_f16(d);
        std::memcpy(ob, &dh, 2);
        for (int j = 0; j < 32; ++j) {
            const float t = xb[j] * id;
            ((int8_t*)(ob + 2))[j] = (int8_t)std::round(t);  // std::round: half away from zero
        }
    }
    return 0;
}

// Q8_0 -> float: x = q * d (ggml to_float, gt_core.cpp:808)
int orc_q8_0_dequantize(const uint8_t* in, int64_t n, float* out) {
    if (n % 32 != 0) return -1;
    for (int64_t blk = 0; blk < n / 32; ++blk) {
        const uint8_t* ib = in + blk * 34;
        uint16_t dh;
        std::memcpy(&dh, ib, 2);
        const float d = f16_to_f32(dh);
        for (int j = 0; j < 32; ++j) out[blk * 32 + j] = (float)((const int8_t*)(ib + 2))[j] * d;
    }
    return 0;
}

// Decode with a Q8_0 K/V cache: the reference's route is k.dequantize(float32), v.dequantize(
// float32) then F.scaled_dot_product_attention(q[B,H,1,D], k, v, is_causal=False)
// (_tensor.py:1188-1196 then gt_ops_nn.cpp:2423). Sequence b attends only its first seq_lens[b]
// cached rows. k_q8/v_q8 hold (B, Hkv, Smax, D) values as rows of D/32 Q8_0 blocks.
int orc_decode_q8_0(const double* q, const uint8_t* k_q8, const uint8_t* v_q8, const int32_t* seq_lens,
                    int64_t B, int64_t H, int64_t Hkv, int64_t Smax, int64_t D,
                    float scale, double* out, int nthreads) {
    if (D % 32 != 0 || Hkv <= 0 || H % Hkv != 0) return -1;
    const int64_t group = H / Hkv;
    if (scale <= 0.0f) scale = 1.0f / std::sqrt((float)D);
    const int64_t row_bytes = D / 32 * 34;
    set_threads(nthreads);
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int64_t b = 0; b < B; ++b) {
        for (int64_t h = 0; h < H; ++h) {
            const int64_t hk = h / group;
            const int64_t Lb = std::min<int64_t>(std::max<int32_t>(seq_lens[b], 0), Smax);
            std::vector<float> kr(D), vr(D);
            std::vector<double> sc(Lb);
            const double* qr = q + (b * H + h) * D;
            double mx = -std::numeric_limits<double>::infinity();
            for (int64_t s = 0; s < Lb; ++s) {
                orc_q8_0_dequantize(k_q8 + ((b * Hkv + hk) * Smax + s) * row_bytes, D, kr.data());
                double dot = 0.0;
                for (int64_t d = 0; d < D; ++d) dot += qr[d] * (double)kr[d];
                dot *= (double)scale;
                sc[s] = dot;
                mx = std::max(mx, dot);
            }
            double se = 0.0;
            for (int64_t s = 0; s < Lb; ++s) { sc[s] = std::exp(sc[s] - mx); se += sc[s]; }
            const double inv = se > 0.0 ? 1.0 / se : 0.0;
            double* orow = out + (b * H + h) * D;
            for (int64_t d = 0; d < D; ++d) orow[d] = 0.0;
            for (int64_t s = 0; s < Lb; ++s) {
                const double p = sc[s] * inv;
                if (p == 0.0) continue;
                orc_q8_0_dequantize(v_q8 + ((b * Hkv + hk) * Smax + s) * row_bytes, D, vr.data());
                for (int64_t d = 0; d < D; ++d) orow[d] += p * (double)vr[d];
            }
        }
    }
    return 0;
}

int orc_num_threads(void) { return set_threads(0); }

}  // extern "C"
