// host_experts.cpp — the host expert pool (host_experts.hpp) and its C entry points.
//
// The work of one job is the reference's two phases (host_experts.rs:827-923): phase A computes
// gate and up of every expert in the job straight into the activation, phase B the down rows
// once every activation row exists; the caller's sync folds the experts in router order
// (host_experts.rs:746-760: dst = 0, dst += w * part). What differs is the unit and the layout:
// a unit is one 16-row tile-row of one expert's matrix, read from the packed (tensor-core
// fragment order) banks the GPU fetches from, so the host needs no second copy of an offloaded
// block. Threads claim units from an atomic cursor; the thread that calls sync works too.
//
// Packed tile (16 rows r0..r0+15 x 64 columns = blocks b0, b0+1), as moearc_x_moe_pack writes it:
//   bytes [16 l, 16 l + 16) for l = 4 r + q (r < 8, q < 4): qs bytes 4q..4q+3 of row r block
//   b0, of row r+8 block b0, of row r block b0+1, of row r+8 block b0+1 (byte j: element j in
//   the low nibble, element j + 16 in the high one); then the scales of rows r, r+8 for b0, b0+1
//   at 512 + 4 r (MXFP4, e8m0) or 512 + 8 r (Q4_0, f16) in that order.
// The portable row kernel keeps the reference's f32 arithmetic and order per row and block
// (dot_mxfp4, host_experts.rs:1088-1103: elements 0..15 of the low and of the high half summed
// apart, their sum scaled once per block). The AVX2 kernel takes the input in int16 with a scale
// per 16 elements (relative error below 2^-16 of each group's largest value) so that the weight
// nibbles multiply through vpmaddwd in exact integer arithmetic: about twice the portable f32
// kernel's rate per core.
#include "host_experts.hpp"

#include <immintrin.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <climits>
#include <cmath>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <thread>
#include <vector>

#include "../../include/moearc.h"

namespace moearc {

namespace {

constexpr int OK_ = 0, ERR_ = -1, ERR_ARG_ = -2;
constexpr int T_MXFP4_ = 39, T_Q4_0_ = 2;
constexpr unsigned MAX_JOB_EXPERTS = 32;

// MXFP4 element values doubled (the e8m0 scale below is halved to match) and Q4_0's q - 8.
alignas(16) const int8_t LUT_MXFP4[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
alignas(16) const int8_t LUT_Q4_0[16] = {-8, -7, -6, -5, -4, -3, -2, -1, 0, 1, 2, 3, 4, 5, 6, 7};

// 2^(e - 128): the e8m0 scale times one half (e = 0, 1 give the subnormals 2^-128, 2^-127).
float e8m0_half(uint8_t e) {
    const uint32_t bits = e < 2 ? (0x00200000u << e) : ((uint32_t)(e - 1) << 23);
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t bits;
    if (ex == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            int e = -1;
            uint32_t m = man;
            do {
                m <<= 1;
                ++e;
            } while (!(m & 0x400u));
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (ex == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((ex + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

struct scale_table {
    float v[256];
    scale_table() {
        for (int i = 0; i < 256; ++i) v[i] = e8m0_half((uint8_t)i);
    }
};
const scale_table E8M0;

inline float tile_scale(int wt, const uint8_t *tile, int r, int i) {
    if (wt == T_MXFP4_) return E8M0.v[tile[512 + 4 * r + i]];
    const uint8_t *p = tile + 512 + 8 * r + 2 * i;
    return half_to_float((uint16_t)(p[0] | (p[1] << 8)));
}

// out[R] = sum over the nkt tiles (tile t at first + t * step) of tile_t . x[64 t .. 64 t + 63],
// R = 0..15.
void rows16_scalar(int wt, const uint8_t *first, size_t step, int nkt, const float *x, float *out) {
    const int8_t *lut = wt == T_MXFP4_ ? LUT_MXFP4 : LUT_Q4_0;
    float acc[16] = {};
    for (int t = 0; t < nkt; ++t) {
        const uint8_t *tile = first + (size_t)t * step;
        const float *xk = x + 64 * t;
        for (int R = 0; R < 16; ++R) {
            const int r = R & 7, hi = R >> 3;
            for (int b = 0; b < 2; ++b) {
                float lo = 0.f, up = 0.f;
                for (int q = 0; q < 4; ++q) {
                    const uint8_t *p = tile + (4 * r + q) * 16 + hi * 4 + b * 8;
                    for (int j = 0; j < 4; ++j) {
                        const int el = 4 * q + j;
                        lo += (float)lut[p[j] & 15] * xk[32 * b + el];
                        up += (float)lut[p[j] >> 4] * xk[32 * b + 16 + el];
                    }
                }
                acc[R] += tile_scale(wt, tile, r, 2 * b + hi) * (lo + up);
            }
        }
    }
    std::memcpy(out, acc, sizeof(acc));
}

// An input vector in the AVX2 kernel's form: each 16-element group g quantised to int16 with its
// own scale (q = round(x * 32767 / max|x|), x ~ q * scale), laid out so that one 32-byte load
// pairs with one lane's decoded nibbles: per 64-column tile t and lane column q, the low-nibble
// vector holds elements 64t + 4q .. +3 (twice: rows r and r+8) then 64t + 32 + 4q .. +3 (twice),
// the high-nibble vector the same 16 further on; per tile, the scales as [g 4t x4 | g 4t+2 x4]
// (low) and [g 4t+1 x4 | g 4t+3 x4] (high). The relative error of a group's values is below
// 2^-16 of its largest, far inside the f32 check tolerance of 1e-4.
struct qvec {
    std::vector<int16_t> v;  // [tile][q][lo, hi][16]
    std::vector<float> sc;   // [tile][lo, hi][8]
    std::vector<float> gs;   // [group] scale
    void resize(int n) {
        v.resize((size_t)n * 2);
        sc.resize((size_t)n / 64 * 16);
        gs.resize((size_t)n / 16);
    }
};

// Quantise 16 values (group g of the vector) into q.
void quantise_group(qvec &q, int g, const float *x16) {
    float m = 0.f;
    for (int i = 0; i < 16; ++i) m = std::fmax(m, std::fabs(x16[i]));
    const float inv = m > 0.f ? 32767.f / m : 0.f;
    q.gs[g] = m > 0.f ? m / 32767.f : 0.f;
    const int t = g / 4, part = g % 4;  // part: 0 b0 low, 1 b0 high, 2 b1 low, 3 b1 high
    const int hi = part & 1, b = part >> 1;
    for (int i = 0; i < 16; ++i) {
        const int qc = i / 4, j = i % 4;  // element 4 qc + j of the half-block
        long r = std::lrint(x16[i] * inv);
        r = r > 32767 ? 32767 : (r < -32767 ? -32767 : r);
        int16_t *vec = q.v.data() + (((size_t)t * 4 + qc) * 2 + hi) * 16;
        vec[8 * b + j] = (int16_t)r;      // row r
        vec[8 * b + 4 + j] = (int16_t)r;  // row r + 8
    }
    float *sc = q.sc.data() + ((size_t)t * 2 + hi) * 8 + 4 * b;
    for (int i = 0; i < 4; ++i) sc[i] = q.gs[g];
}

// out[R] = sum over the nkt tiles of tile_t . x with AVX2: per lane l = 4 r + q the 16 packed
// bytes decode through a byte shuffle to 16 low- and 16 high-nibble values, widen to int16 and
// multiply-add against the lane's int16 x vectors (vpmaddwd: products of adjacent elements summed
// in int32, exact); per (tile, r) the four lanes' int32 sums are converted once and scaled by
// weight scale x group scale into [row r | row r+8] float accumulators.
__attribute__((target("avx2,fma,f16c"))) void rows16_avx2(int wt, const uint8_t *first, size_t step, int nkt,
                                                         const qvec &xq, float *out) {
    const __m128i lut = _mm_load_si128(reinterpret_cast<const __m128i *>(wt == T_MXFP4_ ? LUT_MXFP4 : LUT_Q4_0));
    const __m128i m4 = _mm_set1_epi8(0x0F);
    const __m256i dup = _mm256_setr_epi32(0, 0, 1, 1, 2, 2, 3, 3);
    __m256 acc[8];
    for (int r = 0; r < 8; ++r) acc[r] = _mm256_setzero_ps();
    for (int t = 0; t < nkt; ++t) {
        const uint8_t *tile = first + (size_t)t * step;
        const __m256i *xv = reinterpret_cast<const __m256i *>(xq.v.data() + (size_t)t * 4 * 2 * 16);
        const __m256 sxl = _mm256_loadu_ps(xq.sc.data() + (size_t)t * 16);
        const __m256 sxh = _mm256_loadu_ps(xq.sc.data() + (size_t)t * 16 + 8);
        for (int r = 0; r < 8; ++r) {
            __m128 d4;
            if (wt == T_MXFP4_) {
                const uint8_t *e = tile + 512 + 4 * r;
                d4 = _mm_setr_ps(E8M0.v[e[0]], E8M0.v[e[1]], E8M0.v[e[2]], E8M0.v[e[3]]);
            } else {
                d4 = _mm_cvtph_ps(_mm_loadl_epi64(reinterpret_cast<const __m128i *>(tile + 512 + 8 * r)));
            }
            // [d(r,b0) x2 | d(r+8,b0) x2 | d(r,b1) x2 | d(r+8,b1) x2]
            const __m256 sw = _mm256_permutevar8x32_ps(_mm256_castps128_ps256(d4), dup);
            __m256i lo32 = _mm256_setzero_si256(), hi32 = _mm256_setzero_si256();
            for (int q = 0; q < 4; ++q) {
                const __m128i v = _mm_loadu_si128(reinterpret_cast<const __m128i *>(tile + 16 * (4 * r + q)));
                const __m128i lo = _mm_shuffle_epi8(lut, _mm_and_si128(v, m4));
                const __m128i hi = _mm_shuffle_epi8(lut, _mm_and_si128(_mm_srli_epi16(v, 4), m4));
                lo32 = _mm256_add_epi32(lo32, _mm256_madd_epi16(_mm256_cvtepi8_epi16(lo), _mm256_loadu_si256(xv + 2 * q)));
                hi32 = _mm256_add_epi32(hi32, _mm256_madd_epi16(_mm256_cvtepi8_epi16(hi), _mm256_loadu_si256(xv + 2 * q + 1)));
            }
            acc[r] = _mm256_fmadd_ps(_mm256_cvtepi32_ps(lo32), _mm256_mul_ps(sw, sxl), acc[r]);
            acc[r] = _mm256_fmadd_ps(_mm256_cvtepi32_ps(hi32), _mm256_mul_ps(sw, sxh), acc[r]);
        }
    }
    for (int r = 0; r < 8; ++r) {
        alignas(32) float v[8];
        _mm256_store_ps(v, acc[r]);
        out[r] = (v[0] + v[1]) + (v[4] + v[5]);
        out[r + 8] = (v[2] + v[3]) + (v[6] + v[7]);
    }
}

inline float act_fn(int act, float g, float u, float alpha, float limit) {
    if (act == 1) {
        const float xg = std::fmin(g, limit);
        const float yu = std::fmin(std::fmax(u, -limit), limit);
        return (xg / (1.0f + std::exp(alpha * (-xg)))) * (yu + 1.0f);
    }
    return (g / (1.0f + std::exp(-g))) * u;
}

bool cpu_has_avx2() {
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") && __builtin_cpu_supports("f16c");
}

uint64_t now_ns() {
    return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

}  // namespace

// One worker's acknowledgement of the last job it finished, on a cache line of its own.
struct alignas(64) ack_word {
    std::atomic<uint64_t> v{0};
};

struct host_pool {
    int n_threads = 0;
    bool avx2 = false;
    std::vector<std::thread> threads;
    // A job's result is complete when all its units are done (done_b); the next submit rewrites
    // the job only once every worker has acknowledged the previous epoch, so a worker that comes
    // late to a job (descheduled, or waking from sleep) never reads a half-written one, and sync
    // never waits for a worker that has nothing left to do.
    std::vector<ack_word> acks;
    std::atomic<bool> stop{false};
    std::atomic<uint64_t> epoch{0};  // bumped once per job: workers run the job of the new epoch
    std::mutex mu;
    std::condition_variable cv;
    // the job, written by host_submit before the epoch bump
    host_shape s{};
    const uint8_t *gu = nullptr, *dn = nullptr;
    size_t gu_stride = 0, dn_stride = 0;
    unsigned n = 0;
    unsigned ids[MAX_JOB_EXPERTS] = {};
    float weights[MAX_JOB_EXPERTS] = {};
    std::vector<float> x, act, part;  // x [H], act [32][I], part [32][H]
    qvec xq;                          // x in the AVX2 kernel's form
    std::vector<qvec> actq;           // each expert's activation in that form (AVX2)
    long units_a = 0, units_b = 0;
    std::atomic<long> cursor_a{0}, cursor_b{0}, done_a{0}, done_b{0};
    bool pending = false;
    std::atomic<unsigned long long> jobs{0}, experts{0}, busy_ns{0}, wait_ns{0};

    // Phase A unit u: expert u / (I/16), tile-row u % (I/16) of gate and up -> 16 activations
    // (and, for the AVX2 kernel, their quantised group).
    void unit_a(long u) {
        const int ntr = s.I / 16, nkt = s.H / 64, tb = s.wtype == T_MXFP4_ ? 544 : 576;
        const int i = (int)(u / ntr), tr = (int)(u % ntr);
        const uint8_t *base = gu + (size_t)ids[i] * gu_stride + (size_t)tr * nkt * 2 * tb;
        float g[16], up[16];
        if (avx2) {
            rows16_avx2(s.wtype, base, (size_t)2 * tb, nkt, xq, g);
            rows16_avx2(s.wtype, base + tb, (size_t)2 * tb, nkt, xq, up);
        } else {
            rows16_scalar(s.wtype, base, (size_t)2 * tb, nkt, x.data(), g);
            rows16_scalar(s.wtype, base + tb, (size_t)2 * tb, nkt, x.data(), up);
        }
        float *a = act.data() + (size_t)i * s.I + tr * 16;
        for (int r = 0; r < 16; ++r) a[r] = act_fn(s.act, g[r], up[r], s.alpha, s.limit);
        if (avx2) quantise_group(actq[i], tr, a);
    }

    // Phase B unit u: expert u / (H/16), tile-row u % (H/16) of down -> 16 output rows.
    void unit_b(long u) {
        const int ntr = s.H / 16, nkt = s.I / 64, tb = s.wtype == T_MXFP4_ ? 544 : 576;
        const int i = (int)(u / ntr), tr = (int)(u % ntr);
        const uint8_t *base = dn + (size_t)ids[i] * dn_stride + (size_t)tr * nkt * tb;
        float *o = part.data() + (size_t)i * s.H + tr * 16;
        if (avx2)
            rows16_avx2(s.wtype, base, (size_t)tb, nkt, actq[i], o);
        else
            rows16_scalar(s.wtype, base, (size_t)tb, nkt, act.data() + (size_t)i * s.I, o);
    }

    // Claim and run units until both phases' cursors run dry; phase B starts once every phase A
    // unit is done.
    void work() {
        const uint64_t t0 = now_ns();
        long done = 0;
        for (long u; (u = cursor_a.fetch_add(1, std::memory_order_relaxed)) < units_a;) {
            unit_a(u);
            ++done;
        }
        if (done) done_a.fetch_add(done, std::memory_order_acq_rel);
        // every activation row exists before any down row reads it
        while (done_a.load(std::memory_order_acquire) < units_a) {
            if (stop.load(std::memory_order_relaxed)) return;
            _mm_pause();
        }
        done = 0;
        for (long u; (u = cursor_b.fetch_add(1, std::memory_order_relaxed)) < units_b;) {
            unit_b(u);
            ++done;
        }
        if (done) done_b.fetch_add(done, std::memory_order_acq_rel);
        busy_ns.fetch_add(now_ns() - t0, std::memory_order_relaxed);
    }

    void worker(int id) {
        uint64_t seen = 0;
        for (;;) {
            // spin for about 5 ms after a job (a decode step posts one per offloaded block), then
            // sleep until the next one
            const uint64_t idle0 = now_ns();
            for (unsigned i = 0;; ++i) {
                if (stop.load(std::memory_order_acquire)) return;
                const uint64_t e = epoch.load(std::memory_order_acquire);
                if (e != seen) {
                    seen = e;
                    break;
                }
                if ((i & 255) == 255 && now_ns() - idle0 > 5000000) {
                    std::unique_lock<std::mutex> lk(mu);
                    cv.wait(lk, [&] { return stop.load() || epoch.load() != seen; });
                } else {
                    _mm_pause();
                }
            }
            work();
            acks[id].v.store(seen, std::memory_order_release);
        }
    }
};

host_pool *host_pool_create(int n_threads) {
    if (n_threads <= 0) {
        const char *env = std::getenv("MOEARC_HOST_THREADS");
        if (env && std::atoi(env) > 0) {
            n_threads = std::atoi(env);
        } else {
            const long n = sysconf(_SC_NPROCESSORS_ONLN);
            n_threads = n > 1 ? (int)(n - 1) : 1;
        }
    }
    n_threads = std::min(n_threads, 256);
    auto *p = new (std::nothrow) host_pool();
    if (!p) return nullptr;
    p->n_threads = n_threads;
    p->acks = std::vector<ack_word>(n_threads);
    const char *sc = std::getenv("MOEARC_HOST_SCALAR");
    p->avx2 = cpu_has_avx2() && !(sc && sc[0] == '1');
    try {
        for (int i = 0; i < n_threads; ++i) p->threads.emplace_back([p, i] { p->worker(i); });
    } catch (...) {
        host_pool_destroy(p);
        return nullptr;
    }
    return p;
}

void host_pool_destroy(host_pool *p) {
    if (!p) return;
    {
        std::lock_guard<std::mutex> lk(p->mu);
        p->stop.store(true, std::memory_order_release);
    }
    p->cv.notify_all();
    for (auto &t : p->threads) t.join();
    delete p;
}

int host_pool_threads(const host_pool *p) { return p ? p->n_threads : 0; }

size_t host_packed_bytes(const host_shape &s, int which) {
    if (s.H <= 0 || s.I <= 0 || s.H % 64 || s.I % 64 || (s.wtype != T_MXFP4_ && s.wtype != T_Q4_0_)) return 0;
    const size_t blocks = (size_t)s.H * s.I / 32, bb = s.wtype == T_MXFP4_ ? 17 : 18;
    return which == 0 ? 2 * blocks * bb : blocks * bb;
}

int host_submit(host_pool *p, const host_shape &s, const uint8_t *gu, const uint8_t *dn, const unsigned *ids,
                const float *weights, unsigned n, const float *x) {
    if (!p || !x || (n && (!gu || !dn || !ids || !weights))) return ERR_;
    if (p->pending) return ERR_;
    if (n > MAX_JOB_EXPERTS || !host_packed_bytes(s, 0) || (s.act != 0 && s.act != 1)) return ERR_ARG_;
    // every worker done with the previous job before it is rewritten
    const uint64_t prev = p->epoch.load(std::memory_order_relaxed);
    for (auto &a : p->acks)
        while (a.v.load(std::memory_order_acquire) != prev) _mm_pause();
    p->s = s;
    p->gu = gu;
    p->dn = dn;
    p->gu_stride = host_packed_bytes(s, 0);
    p->dn_stride = host_packed_bytes(s, 1);
    p->n = n;
    for (unsigned i = 0; i < n; ++i) {
        p->ids[i] = ids[i];
        p->weights[i] = weights[i];
    }
    try {
        p->x.assign(x, x + s.H);
        if (p->act.size() < (size_t)MAX_JOB_EXPERTS * s.I) p->act.resize((size_t)MAX_JOB_EXPERTS * s.I);
        if (p->part.size() < (size_t)MAX_JOB_EXPERTS * s.H) p->part.resize((size_t)MAX_JOB_EXPERTS * s.H);
        if (p->avx2) {
            p->xq.resize(s.H);
            for (int g = 0; g < s.H / 16; ++g) quantise_group(p->xq, g, x + 16 * g);
            if (p->actq.size() < MAX_JOB_EXPERTS) p->actq.resize(MAX_JOB_EXPERTS);
            for (unsigned i = 0; i < n; ++i) p->actq[i].resize(s.I);
        }
    } catch (...) {
        return ERR_;
    }
    p->units_a = (long)n * (s.I / 16);
    p->units_b = (long)n * (s.H / 16);
    p->cursor_a.store(0, std::memory_order_relaxed);
    p->cursor_b.store(0, std::memory_order_relaxed);
    p->done_a.store(0, std::memory_order_relaxed);
    p->done_b.store(0, std::memory_order_relaxed);
    p->pending = true;
    {
        std::lock_guard<std::mutex> lk(p->mu);
        p->epoch.fetch_add(1, std::memory_order_acq_rel);
    }
    p->cv.notify_all();
    p->jobs.fetch_add(1, std::memory_order_relaxed);
    p->experts.fetch_add(n, std::memory_order_relaxed);
    return OK_;
}

int host_sync(host_pool *p, float *out) {
    if (!p || !out) return ERR_;
    if (!p->pending) return ERR_;
    p->work();
    const uint64_t w0 = now_ns();
    while (p->done_b.load(std::memory_order_acquire) < p->units_b) _mm_pause();
    p->wait_ns.fetch_add(now_ns() - w0, std::memory_order_relaxed);
    const int H = p->s.H;
    for (int r = 0; r < H; ++r) out[r] = 0.f;
    for (unsigned i = 0; i < p->n; ++i) {
        const float w = p->weights[i];
        const float *part = p->part.data() + (size_t)i * H;
        for (int r = 0; r < H; ++r) {
            const float t = w * part[r];
            out[r] = out[r] + t;
        }
    }
    p->pending = false;
    return OK_;
}

void host_stats(const host_pool *p, unsigned long long out[4]) {
    out[0] = p ? p->jobs.load() : 0;
    out[1] = p ? p->experts.load() : 0;
    out[2] = p ? p->busy_ns.load() : 0;
    out[3] = p ? p->wait_ns.load() : 0;
}

void host_reset_stats(host_pool *p) {
    if (!p) return;
    p->jobs = 0;
    p->experts = 0;
    p->busy_ns = 0;
    p->wait_ns = 0;
}

}  // namespace moearc

using namespace moearc;

namespace {

bool shape_of(const moearc_x_moe_desc *d, host_shape &s) {
    if (!d) return false;
    s = host_shape{(int)d->n_embd, (int)d->n_ff, (int)d->wtype, (int)d->act, d->alpha, d->limit};
    return host_packed_bytes(s, 0) != 0;
}

// One packed tile from GGUF rows: the layout in the header comment.
void pack_tile(uint8_t *tile, const uint8_t *mat, size_t nb, int bb, int tr, int tk) {
    const int sb = bb - 16, qs_off = bb - 16;
    for (int lane = 0; lane < 32; ++lane) {
        const int r = lane >> 2, q = lane & 3;
        const size_t rowA = (size_t)tr * 16 + r, rowB = rowA + 8, bA = (size_t)tk * 2, bB = bA + 1;
        const uint8_t *src[4] = {mat + (rowA * nb + bA) * bb, mat + (rowB * nb + bA) * bb,
                                 mat + (rowA * nb + bB) * bb, mat + (rowB * nb + bB) * bb};
        uint8_t *o = tile + lane * 16;
        for (int i = 0; i < 4; ++i)
            for (int j = 0; j < 4; ++j) o[4 * i + j] = src[i][qs_off + 4 * q + j];
        if (q == 0)
            for (int i = 0; i < 4; ++i)
                for (int k = 0; k < sb; ++k) tile[512 + r * 4 * sb + i * sb + k] = src[i][k];
    }
}

}  // namespace

extern "C" {

moearc_x_host_pool *moearc_x_host_pool_create(int n_threads) {
    return reinterpret_cast<moearc_x_host_pool *>(host_pool_create(n_threads));
}

void moearc_x_host_pool_destroy(moearc_x_host_pool *p) { host_pool_destroy(reinterpret_cast<host_pool *>(p)); }

int moearc_x_host_pool_threads(const moearc_x_host_pool *p) {
    return host_pool_threads(reinterpret_cast<const host_pool *>(p));
}

int moearc_x_host_submit(moearc_x_host_pool *p, const moearc_x_moe_desc *d, const void *gateup_packed,
                         const void *down_packed, const unsigned int *experts, const float *weights, unsigned int n,
                         const float *x) {
    host_shape s;
    if (!p || !d) return ERR_;
    if (!shape_of(d, s)) return ERR_ARG_;
    return host_submit(reinterpret_cast<host_pool *>(p), s, static_cast<const uint8_t *>(gateup_packed),
                       static_cast<const uint8_t *>(down_packed), experts, weights, n, x);
}

int moearc_x_host_sync(moearc_x_host_pool *p, float *out) { return host_sync(reinterpret_cast<host_pool *>(p), out); }

int moearc_x_host_ffn(moearc_x_host_pool *p, const moearc_x_moe_desc *d, const void *gateup_packed,
                      const void *down_packed, const unsigned int *experts, const float *weights, unsigned int n,
                      const float *x, float *out) {
    if (!out) return ERR_;
    const int rc = moearc_x_host_submit(p, d, gateup_packed, down_packed, experts, weights, n, x);
    return rc ? rc : moearc_x_host_sync(p, out);
}

void moearc_x_host_stats(const moearc_x_host_pool *p, unsigned long long *out4) {
    if (out4) host_stats(reinterpret_cast<const host_pool *>(p), out4);
}

int moearc_x_moe_pack_host(const moearc_x_moe_desc *d, const void *gate, const void *up, const void *down,
                           unsigned int n_expert, void *gateup_packed, void *down_packed) {
    host_shape s;
    if (!d || !gate || !up || !down || !gateup_packed || !down_packed) return ERR_;
    if (!shape_of(d, s)) return ERR_ARG_;
    const int bb = s.wtype == T_MXFP4_ ? 17 : 18, tb = 32 * bb;
    const int ntr_i = s.I / 16, nkt_h = s.H / 64, ntr_h = s.H / 16, nkt_i = s.I / 64;
    const size_t mat_i = (size_t)s.I * s.H / 32 * bb;  // one expert's gate (or up, or down)
    auto *gu = static_cast<uint8_t *>(gateup_packed);
    auto *dn = static_cast<uint8_t *>(down_packed);
    for (unsigned e = 0; e < n_expert; ++e) {
        const uint8_t *g = static_cast<const uint8_t *>(gate) + e * mat_i;
        const uint8_t *u = static_cast<const uint8_t *>(up) + e * mat_i;
        const uint8_t *w = static_cast<const uint8_t *>(down) + e * mat_i;
        uint8_t *ge = gu + e * 2 * mat_i, *de = dn + e * mat_i;
        for (int tr = 0; tr < ntr_i; ++tr)
            for (int tk = 0; tk < nkt_h; ++tk) {
                const size_t t = (size_t)tr * nkt_h + tk;
                pack_tile(ge + (2 * t) * tb, g, (size_t)nkt_h * 2, bb, tr, tk);
                pack_tile(ge + (2 * t + 1) * tb, u, (size_t)nkt_h * 2, bb, tr, tk);
            }
        for (int tr = 0; tr < ntr_h; ++tr)
            for (int tk = 0; tk < nkt_i; ++tk)
                pack_tile(de + ((size_t)tr * nkt_i + tk) * tb, w, (size_t)nkt_i * 2, bb, tr, tk);
    }
    return OK_;
}

}  // extern "C"
