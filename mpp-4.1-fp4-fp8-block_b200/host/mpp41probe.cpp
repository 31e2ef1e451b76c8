// mpp41probe: the reference probe's command line (main.swift:80-162) on top of
// the libmpp41 C ABI. Same flags, same seeded inputs (main.swift:409-413,
// 611-638, generators 2785-2842), same report lines and checksums
// (2754-2770, 2844-2884):
//
//   mpp41probe                  packed-numeric roundtrip checks, PASS / FAIL
//   --benchmark                 big packed matmul rows, 2048^3, tensor cores
//   --mlp-benchmark             gated MLP rows, tokens=128 hidden=1024 intermediate=4096
//   --skip-tensor               accepted (the MTLTensor probe is Metal-only)
//   --accum-probe               accepted (Apple accumulator probe, not applicable)
//   --iterations N              timed iterations per row (default 20)
//   --mode ref|baseline         MLP rows' inputs: the reference seeds (default) or, for the
//                               MXFP4 rows, BASELINE mode B (x ~ N(0,1), weights N(0,0.02)
//                               quantized OCP-MX on the GPU)
//   --seed N                    seed of the mode-B and new rows' generators (default 0)
//   --w4a4                      W4A4 and NVFP4 layer rows (config-0 shape)
//   --moe                       mixture-of-experts row (T=512 H=7168 I=2048, 32 experts, top-8,
//                               shared expert: one GPU's share of BASELINE config 4)
//   --json                      benchmark rows as JSON lines instead of text
//   --gpus N                    1 only (multi-GPU runs are one process per GPU)
//
// Buffers live in device memory (mpp41_alloc); inputs are generated on the host
// and uploaded, outputs downloaded for the checksums.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <string>
#include <vector>

#include "mpp41.h"

namespace {

// Reference flags (main.swift:80-162, intArgument main.swift:2886-2892): boolean
// switches, and --name=value integers that fall back to their default when
// absent or not a number.
std::vector<std::string> g_args;
bool g_json = false;
bool g_baseline = false;
uint32_t g_seed = 0;

bool has_flag(const char *name)
{
    for (const auto &a : g_args)
        if (a == name) return true;
    return false;
}

long int_arg(const char *name, long def)
{
    const std::string prefix = std::string(name) + "=";
    for (const auto &a : g_args)
        if (a.compare(0, prefix.size(), prefix) == 0) {
            char *end = nullptr;
            const char *v = a.c_str() + prefix.size();
            const long r = strtol(v, &end, 10);
            return (*v && end && !*end) ? r : def;
        }
    return def;
}

// One timed benchmark row.
struct Result {
    std::string name;
    double seconds;   // for `iterations` calls
    int iterations;
    double flops;     // per call
    std::string checksum;
};

// Rows as the reference prints them (printMatmulBenchmarkResult /
// printMLPBenchmarkResult, main.swift:2754-2770) followed by its relative
// slowdown table (main.swift:2772-2783), or one JSON line per row.
void print_results(const std::vector<Result> &rs, const char *unit)
{
    if (rs.empty()) return;
    size_t best = 0;
    for (size_t i = 0; i < rs.size(); ++i) {
        const Result &r = rs[i];
        const double ms = r.seconds * 1e3 / r.iterations, tops = r.flops * r.iterations / r.seconds / 1e12;
        if (g_json)
            printf("{\"row\": \"%s\", \"ms\": %.5f, \"tops\": %.3f, \"checksum\": \"%s\"}\n", r.name.c_str(), ms,
                   tops, r.checksum.c_str());
        else
            printf("  %s:\n    %.3f ms/%s, %.3f effective TOPS\n    checksum: %s\n", r.name.c_str(), ms, unit, tops,
                   r.checksum.c_str());
        if (r.seconds / r.iterations < rs[best].seconds / rs[best].iterations) best = i;
    }
    if (g_json) return;
    const double b = rs[best].seconds / rs[best].iterations;
    printf("  relative slowdown, best = %s:\n", rs[best].name.c_str());
    for (const Result &r : rs) printf("    %s: %.2fx\n", r.name.c_str(), r.seconds / r.iterations / b);
}

[[noreturn]] void die(mpp41_status s, const char *what)
{
    fprintf(stderr, "error: %s: %s (%s)\n", what, mpp41_status_string(s), mpp41_last_error());
    exit(1);
}

void check(mpp41_status s, const char *what)
{
    if (s != MPP41_OK) die(s, what);
}

// ---------------------------------------------------------------- generators
// state = state * 1664525 + 1013904223 + index (wrapping), as the reference.
inline uint32_t lcg(uint32_t state, size_t index) { return state * 1664525u + 1013904223u + (uint32_t)index; }

std::vector<uint8_t> packed_bytes(size_t n, uint32_t seed)
{
    std::vector<uint8_t> v(n);
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) { s = lcg(s, i); v[i] = (uint8_t)(s >> 16); }
    return v;
}

std::vector<uint8_t> pattern_bytes(size_t n, uint32_t seed, const std::vector<uint8_t> &pattern)
{
    std::vector<uint8_t> v(n);
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) { s = lcg(s, i); v[i] = pattern[s % pattern.size()]; }
    return v;
}

std::vector<_Float16> half_values(size_t n, uint32_t seed, float scale = 0.25f)
{
    std::vector<_Float16> v(n);
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) {
        s = lcg(s, i);
        const int nib = (int)((s >> 28) & 0xF);
        v[i] = (_Float16)((float)((nib ^ 8) - 8) * scale);
    }
    return v;
}

// N(0, sigma) by Box-Muller over the same LCG (mode B inputs).
std::vector<float> normal_values(size_t n, uint32_t seed, float sigma)
{
    std::vector<float> v(n);
    uint32_t s = seed;
    for (size_t i = 0; i < n; i += 2) {
        s = lcg(s, i);
        const double u1 = ((s >> 8) + 1.0) / 16777217.0;
        s = lcg(s, i + 1);
        const double u2 = (s >> 8) / 16777216.0;
        const double r = std::sqrt(-2.0 * std::log(u1)), th = 6.283185307179586 * u2;
        v[i] = (float)(r * std::cos(th) * sigma);
        if (i + 1 < n) v[i + 1] = (float)(r * std::sin(th) * sigma);
    }
    return v;
}

std::vector<int8_t> int8_values(size_t n, uint32_t seed)
{
    std::vector<int8_t> v(n);
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) { s = lcg(s, i); v[i] = (int8_t)((int)((s >> 28) & 0xF) ^ 8) - 8; }
    return v;
}

const std::vector<uint8_t> kE4M3Pattern = {0x00, 0x20, 0x30, 0x38, 0x40, 0xb0, 0xb8, 0xc0, 0x58, 0xd8};
const std::vector<uint8_t> kE5M2Pattern = {0x00, 0x34, 0x38, 0x3c, 0x40, 0xb4, 0xb8, 0xbc, 0xc0, 0x64};
const std::vector<uint8_t> kScalePattern = {124, 125, 126, 127, 127, 128, 128, 129, 130};
// MoE row: random E2M1 bytes with block scales 2^-9..2^-5, so that the
// 7168-long gate/up sums and the 2048-long down sums stay well inside fp16
const std::vector<uint8_t> kMoeScalePattern = {118, 119, 120, 121, 122};

// ---------------------------------------------------------------- checksums
// 32 samples at stride count/32 (main.swift:2844-2884)
std::string float_checksum(const float *p, size_t n)
{
    const size_t step = n / 32 ? n / 32 : 1;
    double sum = 0;
    int samples = 0;
    for (size_t i = 0; i < n; i += step) { sum += p[i]; ++samples; }
    char buf[96];
    snprintf(buf, sizeof(buf), "%.6g over %d samples", sum, samples);
    return buf;
}

std::string int_checksum(const int32_t *p, size_t n)
{
    const size_t step = n / 32 ? n / 32 : 1;
    long long sum = 0;
    int samples = 0;
    for (size_t i = 0; i < n; i += step) { sum += p[i]; ++samples; }
    return std::to_string(sum) + " over " + std::to_string(samples) + " samples";
}

std::string half_raw_checksum(const uint16_t *p, size_t n)
{
    const size_t step = n / 32 ? n / 32 : 1;
    unsigned long long sum = 0;
    int samples = 0;
    for (size_t i = 0; i < n; i += step) { sum += p[i]; ++samples; }
    return "raw16 sum " + std::to_string(sum) + " over " + std::to_string(samples) + " samples";
}

// ---------------------------------------------------------------- device buffers
struct Dev {
    mpp41_ctx *ctx = nullptr;
    void *p = nullptr;
    size_t n = 0;
    Dev(mpp41_ctx *c, size_t bytes) : ctx(c), n(bytes) { if (bytes) check(mpp41_alloc(c, bytes, &p), "alloc"); }
    template <class T> Dev(mpp41_ctx *c, const std::vector<T> &host) : Dev(c, host.size() * sizeof(T))
    {
        if (n) check(mpp41_upload(ctx, p, host.data(), n), "upload");
    }
    ~Dev() { if (p) mpp41_free(ctx, p); }
    Dev(const Dev &) = delete;
    Dev &operator=(const Dev &) = delete;
    template <class T> std::vector<T> get() const
    {
        std::vector<T> h(n / sizeof(T));
        check(mpp41_download(ctx, h.data(), p, n), "download");
        return h;
    }
};

// ---------------------------------------------------------------- roundtrip KATs
struct Case {
    const char *name, *kernel;
    std::vector<float> in, expected;
};

bool run_roundtrips(mpp41_ctx *ctx)
{
    const std::vector<Case> cases = {
        {"FP4 E2M1", "fp4_e2m1_roundtrip",
         {-8, -6, -4, -3, -2, -1.5f, -1, -0.5f, 0, 0.5f, 1, 1.5f, 2, 3, 4, 8},
         {-6, -6, -4, -3, -2, -1.5f, -1, -0.5f, 0, 0.5f, 1, 1.5f, 2, 3, 4, 6}},
        {"FP8 E4M3", "fp8_e4m3_roundtrip", {-512, -448, -16, -0.5f, 0, 0.125f, 16, 512},
         {-448, -448, -16, -0.5f, 0, 0.125f, 16, 448}},
        {"FP8 E5M2", "fp8_e5m2_roundtrip", {-57344, -1024, -2, -0.5f, 0, 0.25f, 1024, 57344},
         {-57344, -1024, -2, -0.5f, 0, 0.25f, 1024, 57344}},
    };
    bool all = true;
    for (const Case &c : cases) {
        Dev in(ctx, c.in), packed(ctx, 16), out(ctx, c.in.size() * sizeof(float));
        check(mpp41_roundtrip(ctx, c.kernel, static_cast<const float *>(in.p), static_cast<uint8_t *>(packed.p),
                              static_cast<float *>(out.p)),
              c.kernel);
        check(mpp41_synchronize(ctx), "synchronize");
        const std::vector<float> got = out.get<float>();
        bool ok = true;
        for (size_t i = 0; i < got.size(); ++i) ok = ok && std::fabs(got[i] - c.expected[i]) <= 1e-5f;
        all = all && ok;
        printf("%s: %s\n", c.name, ok ? "pass" : "FAIL");
        printf("  input:    ");
        for (float v : c.in) printf("%g ", v);
        printf("\n  unpacked: ");
        for (float v : got) printf("%g ", v);
        printf("\n");
    }
    return all;
}

// ---------------------------------------------------------------- big matmul rows
template <class F>
double time_calls(mpp41_ctx *ctx, int iterations, F call)
{
    call();   // warm-up
    check(mpp41_synchronize(ctx), "warm-up");
    check(mpp41_timer_start(ctx), "timer");
    for (int i = 0; i < iterations; ++i) call();
    double sec = 0;
    check(mpp41_timer_stop(ctx, &sec), "timer");
    check(mpp41_synchronize(ctx), "timed calls");
    return sec;
}

void run_big_matmul(mpp41_ctx *ctx)
{
    const long size = int_arg("--matmul-size", 2048);
    const uint32_t M = (uint32_t)int_arg("--m", size), N = (uint32_t)int_arg("--n", size), K = (uint32_t)int_arg("--k", size);
    const int iters = (int)int_arg("--iterations", 3);
    if ((long)M <= 0 || (long)N <= 0 || (long)K <= 0 || iters <= 0) {
        fprintf(stderr, "error: Matmul sizes and iterations must be positive.\n");
        exit(1);
    }
    const bool sweep = has_flag("--fp4-group-sweep");
    if (!g_json) {
        printf("\nBig packed matmul benchmark:\n");
        printf("  shape: A %ux%u, B %ux%u, C %ux%u\n", M, K, K, N, M, N);
        printf("  iterations: %d\n", iters);
        if (sweep) printf("  FP4 unpack group sweep: 8 and 16 elements\n");
    }
    const auto a_packed = packed_bytes((size_t)M * K / 2, 0x12345678u);
    const auto b_packed = packed_bytes((size_t)N * K / 2, 0x87654321u);
    const auto a_half = half_values((size_t)M * K, 0x2468ace0u);
    const auto a_int8 = int8_values((size_t)M * K, 0x13579bdfu);
    const auto b_half = half_values((size_t)N * K, 0xfdb97531u, 0.03125f);
    Dev dap(ctx, a_packed), dbp(ctx, b_packed), dah(ctx, a_half), dai(ctx, a_int8), dbh(ctx, b_half);
    struct Row { const char *name, *kernel; const Dev *a, *b; int out; bool sweep_only; };   // out: 0 f32, 1 half, 2 i32
    // the reference's order: FP4, the g8 sweep rows, then the others (main.swift:580)
    const Row rows[] = {
        {"FP4 E2M1 g16 -> FP32 accumulate", "fp4_e2m1_matmul_benchmark", &dap, &dbp, 0, false},
        {"FP4 E2M1 g8 -> FP32 accumulate", "fp4_e2m1_matmul_g8_benchmark", &dap, &dbp, 0, true},
        {"half x FP4 E2M1 g8 -> half accumulate", "half_fp4_matmul_half_g8_benchmark", &dah, &dbp, 1, true},
        {"half x FP4 E2M1 g16 -> half accumulate", "half_fp4_matmul_half_benchmark", &dah, &dbp, 1, false},
        {"half x INT4 -> half accumulate", "half_int4_matmul_half_benchmark", &dah, &dbp, 1, false},
        {"INT8 x half -> half accumulate", "int8_half_matmul_half_benchmark", &dai, &dbh, 1, false},
        {"INT4 x INT4 -> INT32 accumulate", "int4_int8_matmul_benchmark", &dap, &dbp, 2, false},
    };
    const mpp41_matmul_config cfg = {M, N, K, K / 2};
    std::vector<Result> results;
    for (const Row &r : rows) {
        if (r.sweep_only && !sweep) continue;
        Dev c(ctx, (size_t)M * N * (r.out == 1 ? 2 : 4));
        Dev ws(ctx, mpp41_matmul_workspace_bytes(r.kernel, &cfg));
        const double sec = time_calls(ctx, iters, [&] {
            check(mpp41_matmul(ctx, r.kernel, r.a->p, r.b->p, c.p, &cfg, ws.p), r.kernel);
        });
        std::string cks;
        if (r.out == 0) { const auto h = c.get<float>(); cks = float_checksum(h.data(), h.size()); }
        else if (r.out == 1) { const auto h = c.get<uint16_t>(); cks = half_raw_checksum(h.data(), h.size()); }
        else { const auto h = c.get<int32_t>(); cks = int_checksum(h.data(), h.size()); }
        results.push_back({r.name, sec, iters, 2.0 * M * N * (double)K, cks});
    }
    print_results(results, "matmul");
}

std::vector<_Float16> to_half(const std::vector<float> &v)
{
    std::vector<_Float16> h(v.size());
    for (size_t i = 0; i < v.size(); ++i) h[i] = (_Float16)v[i];
    return h;
}

// OCP-MX MXFP4 weights [rows][depth] quantized on the GPU from N(0, 0.02).
struct MxWeights {
    Dev q, s;
    MxWeights(mpp41_ctx *ctx, uint32_t rows, uint32_t depth, uint32_t seed)
        : q(ctx, (size_t)rows * depth / 2), s(ctx, (size_t)rows * depth / 32)
    {
        Dev w(ctx, normal_values((size_t)rows * depth, seed, 0.02f));
        check(mpp41_quantize_mxfp4(ctx, (const float *)w.p, rows, depth, (uint8_t *)q.p, (uint8_t *)s.p), "quantize");
        check(mpp41_synchronize(ctx), "quantize");
    }
};

// NVFP4 weights (E2M1 + UE4M3 per 16 + fp32 tensor scale) quantized on the GPU from N(0, 0.02).
struct NvWeights {
    Dev q, s, t;
    NvWeights(mpp41_ctx *ctx, uint32_t rows, uint32_t depth, uint32_t seed)
        : q(ctx, (size_t)rows * depth / 2), s(ctx, (size_t)rows * depth / 16), t(ctx, 4)
    {
        Dev w(ctx, normal_values((size_t)rows * depth, seed, 0.02f));
        check(mpp41_quantize_nvfp4(ctx, (const float *)w.p, rows, depth, (uint8_t *)q.p, (uint8_t *)s.p, (float *)t.p),
              "quantize NVFP4");
        check(mpp41_synchronize(ctx), "quantize NVFP4");
    }
};

// ---------------------------------------------------------------- W4A4 / NVFP4 rows (no reference counterpart)
void run_w4a4(mpp41_ctx *ctx)
{
    const uint32_t T = 128, H = 1024, I = 4096;
    if (!g_json) printf("\nW4A4 MLP rows (activations quantized too, FP4 tensor cores):\n  shape: tokens=%u, hidden=%u, intermediate=%u\n", T, H, I);
    Dev x(ctx, to_half(normal_values((size_t)T * H, 0x5A5A0000u ^ g_seed, 1.0f)));
    MxWeights g(ctx, I, H, 0x5A5A0001u ^ g_seed), u(ctx, I, H, 0x5A5A0002u ^ g_seed), d(ctx, H, I, 0x5A5A0003u ^ g_seed);
    Dev out(ctx, (size_t)T * H * 2), scratch(ctx, mpp41_mlp_w4a4_scratch_bytes(T, H, I));
    const int iters = (int)int_arg("--mlp-iterations", 3);
    std::vector<Result> results;
    double sec = time_calls(ctx, iters, [&] {
        check(mpp41_mlp_w4a4(ctx, T, H, I, x.p, (const uint8_t *)g.q.p, (const uint8_t *)g.s.p, (const uint8_t *)u.q.p,
                             (const uint8_t *)u.s.p, (const uint8_t *)d.q.p, (const uint8_t *)d.s.p, out.p, 1, scratch.p),
              "mpp41_mlp_w4a4");
    });
    results.push_back({"W4A4 MXFP4 MLP: x -> MXFP4, kind::mxf4 gate/up + SwiGLU -> MXFP4 mid, kind::mxf4 down", sec, iters,
                       6.0 * T * H * (double)I, half_raw_checksum(out.get<uint16_t>().data(), (size_t)T * H)});
    // NVFP4: weights from the same fp32 values, quantized NVFP4 on the GPU
    NvWeights ng(ctx, I, H, 0x5A5A0001u ^ g_seed), nu(ctx, I, H, 0x5A5A0002u ^ g_seed), nd(ctx, H, I, 0x5A5A0003u ^ g_seed);
    Dev nscr(ctx, mpp41_mlp_nvfp4_scratch_bytes(T, H, I));
    sec = time_calls(ctx, iters, [&] {
        check(mpp41_mlp_nvfp4(ctx, T, H, I, x.p, (const uint8_t *)ng.q.p, (const uint8_t *)ng.s.p, (const float *)ng.t.p,
                              (const uint8_t *)nu.q.p, (const uint8_t *)nu.s.p, (const float *)nu.t.p, (const uint8_t *)nd.q.p,
                              (const uint8_t *)nd.s.p, (const float *)nd.t.p, out.p, 1, nscr.p),
              "mpp41_mlp_nvfp4");
    });
    results.push_back({"W4A4 NVFP4 MLP: E2M1 + UE4M3/16 + fp32 tensor scales, kind::mxf4nvf4", sec, iters,
                       6.0 * T * H * (double)I, half_raw_checksum(out.get<uint16_t>().data(), (size_t)T * H)});
    print_results(results, "MLP");
}

// ---------------------------------------------------------------- MoE row (no reference counterpart)
void run_moe(mpp41_ctx *ctx)
{
    const mpp41_moe_desc d = {512, 7168, 2048, 32, 8, 2048, 1};
    if (!g_json)
        printf("\nMixture-of-experts row (W4A4 experts):\n  shape: tokens=%u, hidden=%u, expert intermediate=%u, "
               "experts=%u, top-%u, shared intermediate=%u\n", d.tokens, d.hidden, d.intermediate, d.experts, d.top_k,
               d.shared_intermediate);
    const size_t H = d.hidden, I = d.intermediate, E = d.experts, Is = d.shared_intermediate;
    Dev x(ctx, to_half(normal_values((size_t)d.tokens * H, 0x3E3E0000u ^ g_seed, 1.0f)));
    Dev logits(ctx, normal_values((size_t)d.tokens * E, 0x3E3E0001u ^ g_seed, 1.0f));
    Dev wg(ctx, packed_bytes(E * I * H / 2, 0x3E3E0002u ^ g_seed)), wu(ctx, packed_bytes(E * I * H / 2, 0x3E3E0003u ^ g_seed));
    Dev wd(ctx, packed_bytes(E * H * I / 2, 0x3E3E0004u ^ g_seed));
    Dev sg(ctx, pattern_bytes(E * I * H / 32, 0x3E3E0005u, kMoeScalePattern)), su(ctx, pattern_bytes(E * I * H / 32, 0x3E3E0006u, kMoeScalePattern));
    Dev sd(ctx, pattern_bytes(E * H * I / 32, 0x3E3E0007u, kMoeScalePattern));
    Dev swg(ctx, packed_bytes(Is * H / 2, 0x3E3E0008u)), swu(ctx, packed_bytes(Is * H / 2, 0x3E3E0009u));
    Dev swd(ctx, packed_bytes(H * Is / 2, 0x3E3E000Au));
    Dev ssg(ctx, pattern_bytes(Is * H / 32, 0x3E3E000Bu, kMoeScalePattern)), ssu(ctx, pattern_bytes(Is * H / 32, 0x3E3E000Cu, kMoeScalePattern));
    Dev ssd(ctx, pattern_bytes(H * Is / 32, 0x3E3E000Du, kMoeScalePattern));
    Dev out(ctx, (size_t)d.tokens * H * 2), scratch(ctx, mpp41_moe_scratch_layout(&d, nullptr));
    auto u8 = [](const Dev &b) { return (const uint8_t *)b.p; };
    const int iters = (int)int_arg("--mlp-iterations", 3);
    const double sec = time_calls(ctx, iters, [&] {
        check(mpp41_moe_w4a4(ctx, &d, x.p, (const float *)logits.p, u8(wg), u8(sg), u8(wu), u8(su), u8(wd), u8(sd), u8(swg),
                             u8(ssg), u8(swu), u8(ssu), u8(swd), u8(ssd), out.p, scratch.p),
              "mpp41_moe_w4a4");
    });
    print_results({{"MoE W4A4: route top-8, grouped kind::mxf4 experts, shared expert, combine", sec, iters,
                    6.0 * d.tokens * H * (double)(d.top_k * I + Is),
                    half_raw_checksum(out.get<uint16_t>().data(), (size_t)d.tokens * H)}},
                  "MLP");
}

// ---------------------------------------------------------------- MLP rows
void run_mlp(mpp41_ctx *ctx)
{
    const long t_arg = int_arg("--mlp-tokens", 128), h_arg = int_arg("--mlp-hidden", 1024);
    const long i_arg = int_arg("--mlp-intermediate", 4 * h_arg), it_arg = int_arg("--mlp-iterations", 3);
    if (t_arg <= 0 || h_arg <= 0 || i_arg <= 0 || it_arg <= 0) {
        fprintf(stderr, "error: MLP dimensions and iterations must be positive.\n");
        exit(1);
    }
    const uint32_t T = (uint32_t)t_arg, H = (uint32_t)h_arg, I = (uint32_t)i_arg;
    const int iters = (int)it_arg;
    const bool sweep = has_flag("--fp4-group-sweep");
    if (!g_json) {
        printf("\nGated MLP benchmark:\n  op: down(silu(gate(x)) * up(x))\n");
        printf("  shape: tokens=%u, hidden=%u, intermediate=%u\n  iterations: %d\n", T, H, I, iters);
        if (g_baseline) printf("  inputs: MXFP4 rows in BASELINE mode B (seed %u)\n", g_seed);
    }
    const size_t gw = (size_t)I * H, dw = (size_t)H * I;
    Dev x_half(ctx, half_values((size_t)T * H, 0x11112222u, 0.125f));
    Dev x_int8(ctx, int8_values((size_t)T * H, 0x22223333u));
    struct Weights { Dev g, u, d; };
    auto halfw = new Weights{{ctx, half_values(gw, 0x55556666u, 0.015625f)}, {ctx, half_values(gw, 0x77778888u, 0.015625f)},
                             {ctx, half_values(dw, 0x9999aaaau, 0.00390625f)}};
    auto i8w = new Weights{{ctx, int8_values(gw, 0x33334444u)}, {ctx, int8_values(gw, 0x44445555u)}, {ctx, int8_values(dw, 0x55557777u)}};
    auto i4w = new Weights{{ctx, packed_bytes(gw / 2, 0x13572468u)}, {ctx, packed_bytes(gw / 2, 0xace01357u)},
                           {ctx, packed_bytes(dw / 2, 0xc001d00du)}};
    auto i2w = new Weights{{ctx, packed_bytes(gw / 4, 0x24681357u)}, {ctx, packed_bytes(gw / 4, 0xbad0cafeu)},
                           {ctx, packed_bytes(dw / 4, 0xd00dc001u)}};
    auto f4w = new Weights{{ctx, packed_bytes(gw / 2, 0xabcd1357u)}, {ctx, packed_bytes(gw / 2, 0x2468bdf0u)},
                           {ctx, packed_bytes(dw / 2, 0x0badcafeu)}};
    auto e4w = new Weights{{ctx, pattern_bytes(gw, 0x11117777u, kE4M3Pattern)}, {ctx, pattern_bytes(gw, 0x22228888u, kE4M3Pattern)},
                           {ctx, pattern_bytes(dw, 0x33339999u, kE4M3Pattern)}};
    auto e5w = new Weights{{ctx, pattern_bytes(gw, 0x4444aaaau, kE5M2Pattern)}, {ctx, pattern_bytes(gw, 0x5555bbbbu, kE5M2Pattern)},
                           {ctx, pattern_bytes(dw, 0x6666ccccu, kE5M2Pattern)}};
    Dev sg(ctx, pattern_bytes((size_t)I * (H / 32), 0x7777ddddu, kScalePattern));
    Dev su(ctx, pattern_bytes((size_t)I * (H / 32), 0x8888eeeeu, kScalePattern));
    Dev sd(ctx, pattern_bytes((size_t)H * (I / 32), 0x9999ffffu, kScalePattern));
    // mode B: x ~ N(0,1) fp16, weights N(0,0.02) quantized OCP-MX on the GPU
    Dev xb(ctx, to_half(normal_values((size_t)T * H, 0x51ED0000u ^ g_seed, 1.0f)));
    MxWeights bg(ctx, I, H, 0x51ED0001u ^ g_seed), bu(ctx, I, H, 0x51ED0002u ^ g_seed), bd(ctx, H, I, 0x51ED0003u ^ g_seed);

    struct Row { const char *name, *kernel; const Weights *w; bool mx; };
    const Row rows[] = {
        {"MPP/NAX MLP half weights: h_h_f + f_h_f", "mpp_mlp_h_h_f_n128", halfw, false},
        {"MPP/NAX MLP INT8 weights: h_i8_f + f_i8_f", "mpp_mlp_h_i8_f_n128", i8w, false},
        {"MPP/NAX MLP INT4 weights: h_i4_f + h_i4_f", "mpp_mlp_h_i4_f_n128", i4w, false},
        {"MPP/NAX MLP FP4 E2M1 weights: h_fp4_f + h_fp4_f", "mpp_mlp_h_fp4_f_n128", f4w, false},
        {"MXFP4 fused MPP 4.1 (native FP4 + E8M0 in-register, n128): h_mxfp4_f", "mxfp4_fused_h_f_n128", f4w, true},
        {"MXFP4 fused MPP 4.1 (native FP4 + E8M0 in-register, n64): h_mxfp4_f", "mxfp4_fused_h_f_n64", f4w, true},
        {"MXFP4 native scale-plane MPP 4.1 (FP4 + E8M0 consumed by matmul2d, n128): h_mxfp4sp_f", "mxfp4_native_sp_h_f_n128", f4w, true},
        {"MXFP4 native scale-plane MPP 4.1 (FP4 + E8M0 consumed by matmul2d, n64): h_mxfp4sp_f", "mxfp4_native_sp_h_f_n64", f4w, true},
        {"MXFP4 host MTLTensor + scale plane (bindless handle, n64): h_mxfp4sph_f", "mxfp4_native_sph_h_f_n64", f4w, true},
        {"MXFP4 coop-input (k64): h_mxfp4ci_f", "mxfp4_fused_ci_h_f_sg_k64", f4w, true},
        {"MXFP4 coop-input (k32): h_mxfp4ci_f", "mxfp4_fused_ci_h_f_sg_k32", f4w, true},
        {"MPP/NAX MLP FP8 E4M3 weights: h_fp8_f + h_fp8_f", "mpp_mlp_h_fp8e4m3_f_n128", e4w, false},
        {"MPP/NAX MLP FP8 E4M3 weights: h_fp8_h + h_fp8_h", "mpp_mlp_h_fp8e4m3_h_n128", e4w, false},
        {"MPP/NAX MLP FP8 E5M2 weights: h_fp8_f + h_fp8_f", "mpp_mlp_h_fp8e5m2_f_n128", e5w, false},
        {"MPP/NAX MLP INT2 weights: h_i2_f + h_i2_f", "mpp_mlp_h_i2_f_n128", i2w, false},
        {"MPP/NAX W8A8 MLP: i8 x int8_t -> i32", "mpp_mlp_i8_i8_i32_n128", i8w, false},
        {"MPP/NAX W4A8 MLP: i8 x int4b -> i32", "mpp_mlp_i8_i4_i32_n128", i4w, false},
        {"MPP/NAX W2A8 MLP: i8 x int2b -> i32", "mpp_mlp_i8_i2_i32_n128", i2w, false},
    };
    const double flops = 2.0 * 3.0 * T * (double)H * I;
    std::vector<Result> results;
    // scalar rows (encodeMLP, main.swift:2575-2634): half x, fp16 mid and out
    Dev smid(ctx, (size_t)T * I * 2), sout(ctx, (size_t)T * H * 2);
    const mpp41_mlp_config scfg = {T, H, I};
    auto scalar_row = [&](const char *name, const char *gate, const char *down, const Weights *w) {
        const double sec = time_calls(ctx, iters, [&] {
            check(mpp41_mlp_scalar(ctx, gate, down, x_half.p, w->g.p, w->u.p, smid.p, w->d.p, sout.p, &scfg), gate);
        });
        const auto h = sout.get<uint16_t>();
        results.push_back({name, sec, iters, flops, half_raw_checksum(h.data(), h.size())});
    };
    scalar_row("half MLP: half x half -> half", "half_mlp_gate_up_benchmark", "half_mlp_down_benchmark", halfw);
    for (const Row &r : rows) {
        mpp41_mlp_desc d;
        check(mpp41_mlp_describe(r.kernel, T, H, I, &d), r.kernel);
        const size_t out_elem = d.out_dtype == MPP41_F16 ? 2 : 4;
        Dev out(ctx, (size_t)T * H * out_elem), scratch(ctx, mpp41_mlp_scratch_bytes(&d));
        const bool mode_b = g_baseline && r.mx;
        const void *x = d.afmt == MPP41_A_S8 ? x_int8.p : (mode_b ? xb.p : x_half.p);
        const void *wg = mode_b ? bg.q.p : r.w->g.p, *wu = mode_b ? bu.q.p : r.w->u.p, *wd = mode_b ? bd.q.p : r.w->d.p;
        const uint8_t *s_g = r.mx ? (const uint8_t *)(mode_b ? bg.s.p : sg.p) : nullptr;
        const uint8_t *s_u = r.mx ? (const uint8_t *)(mode_b ? bu.s.p : su.p) : nullptr;
        const uint8_t *s_d = r.mx ? (const uint8_t *)(mode_b ? bd.s.p : sd.p) : nullptr;
        double sec = 0;
        check(mpp41_mlp_benchmark(ctx, &d, x, wg, wu, wd, s_g, s_u, s_d, scratch.p, out.p, iters, &sec), r.kernel);
        std::string cks;
        if (d.out_dtype == MPP41_S32) { const auto h = out.get<int32_t>(); cks = int_checksum(h.data(), h.size()); }
        else if (d.out_dtype == MPP41_F16) { const auto h = out.get<uint16_t>(); cks = half_raw_checksum(h.data(), h.size()); }
        else { const auto h = out.get<float>(); cks = float_checksum(h.data(), h.size()); }
        results.push_back({r.name, sec, iters, flops, cks});
    }
    scalar_row("half MLP with INT8 weights: half x int8_t -> half", "half_int8_mlp_gate_up_benchmark",
               "half_int8_mlp_down_benchmark", i8w);
    scalar_row("half MLP with INT4 weights: half x int4b_format -> half", "half_int4_mlp_gate_up_benchmark",
               "half_int4_mlp_down_benchmark", i4w);
    scalar_row("half MLP with INT2 weights: half x int2b_format -> half", "half_int2_mlp_gate_up_benchmark",
               "half_int2_mlp_down_benchmark", i2w);
    scalar_row("half MLP with FP4 E2M1 g16 weights: half x FP4 -> half", "half_fp4_mlp_gate_up_benchmark",
               "half_fp4_mlp_down_benchmark", f4w);
    if (sweep)
        scalar_row("half MLP with FP4 E2M1 g8 weights: half x FP4 -> half", "half_fp4_mlp_gate_up_g8_benchmark",
                   "half_fp4_mlp_down_g8_benchmark", f4w);
    print_results(results, "MLP");
    delete halfw; delete i8w; delete i4w; delete i2w; delete f4w; delete e4w; delete e5w;
}

}  // namespace

int main(int argc, char **argv)
{
    // Flags follow the reference command line (main.swift:80-162): booleans by
    // name, integers as --name=value (intArgument, main.swift:2886-2892), and
    // arguments it does not know are ignored. --json, --w4a4, --moe, --seed,
    // --mode and --gpus are this probe's own.
    for (int i = 1; i < argc; ++i) g_args.emplace_back(argv[i]);
    auto value_of = [&](size_t &i, const char *name, std::string &out) {
        const std::string &a = g_args[i];
        const size_t n = strlen(name);
        if (a == name && i + 1 < g_args.size()) { out = g_args[++i]; return true; }
        if (a.compare(0, n, name) == 0 && a.size() > n && a[n] == '=') { out = a.substr(n + 1); return true; }
        return false;
    };
    static const char *const known[] = {"--benchmark", "--mlp-benchmark", "--accum-probe", "--skip-tensor",
                                        "--fp4-group-sweep", "--mxfp4-decompose", "--w4a4", "--moe", "--json"};
    static const char *const known_int[] = {"--matmul-size", "--m", "--n", "--k", "--iterations", "--mlp-tokens",
                                            "--mlp-hidden", "--mlp-intermediate", "--mlp-iterations"};
    for (size_t i = 0; i < g_args.size(); ++i) {
        std::string v;
        if (value_of(i, "--seed", v)) { g_seed = (uint32_t)strtoul(v.c_str(), nullptr, 0); continue; }
        if (value_of(i, "--mode", v)) {
            if (v == "baseline") g_baseline = true;
            else if (v != "ref") { fprintf(stderr, "--mode takes ref or baseline\n"); return 2; }
            continue;
        }
        if (value_of(i, "--gpus", v)) {
            if (atoi(v.c_str()) != 1) {
                fprintf(stderr, "--gpus: this probe drives one GPU; multi-GPU layers run one process per GPU "
                                "(mpp41_comm_init, mpp41_mlp_tp, mpp41_moe_ep)\n");
                return 2;
            }
            continue;
        }
        bool ok = false;
        for (const char *k : known) ok = ok || g_args[i] == k;
        for (const char *k : known_int) {
            const size_t n = strlen(k);
            ok = ok || (g_args[i].compare(0, n, k) == 0 && g_args[i].size() > n && g_args[i][n] == '=');
        }
        if (!ok) fprintf(stderr, "warning: ignoring argument %s\n", g_args[i].c_str());
    }
    g_json = has_flag("--json");
    const bool bench = has_flag("--benchmark"), mlp = has_flag("--mlp-benchmark"), accum = has_flag("--accum-probe");
    const bool w4a4 = has_flag("--w4a4"), moe = has_flag("--moe");
    mpp41_ctx *ctx = nullptr;
    check(mpp41_create(0, &ctx), "mpp41_create");
    char name[256];
    check(mpp41_device_name(ctx, name, sizeof(name)), "device name");
    printf("Device: %s\n", name);
    const bool ok = run_roundtrips(ctx);
    printf("MTLTensor creation probe: not applicable (Metal host API).\n");
    if (bench) run_big_matmul(ctx);
    if (mlp) run_mlp(ctx);
    if (w4a4) run_w4a4(ctx);
    if (moe) run_moe(ctx);
    if (accum) printf("Accumulator precision probe: not applicable (Apple matmul2d semantics).\n");
    if (has_flag("--mxfp4-decompose"))
        printf("MXFP4 decomposition probe: not applicable (Metal kernel-variant timing).\n");
    mpp41_destroy(ctx);
    if (!ok) {
        fprintf(stderr, "error: One or more packed numeric checks failed.\n");
        return 1;
    }
    printf("PASS\n");
    return 0;
}
