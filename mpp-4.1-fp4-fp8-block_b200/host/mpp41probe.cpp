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

int g_iterations = 20;

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
void run_big_matmul(mpp41_ctx *ctx)
{
    const uint32_t M = 2048, N = 2048, K = 2048;
    printf("\nBig packed matmul benchmark:\n");
    printf("  shape: A %ux%u, B %ux%u, C %ux%u\n", M, K, K, N, M, N);
    printf("  iterations: %d\n", g_iterations);
    const auto a_packed = packed_bytes((size_t)M * K / 2, 0x12345678u);
    const auto b_packed = packed_bytes((size_t)N * K / 2, 0x87654321u);
    const auto a_half = half_values((size_t)M * K, 0x2468ace0u);
    const auto a_int8 = int8_values((size_t)M * K, 0x13579bdfu);
    const auto b_half = half_values((size_t)N * K, 0xfdb97531u, 0.03125f);
    Dev dap(ctx, a_packed), dbp(ctx, b_packed), dah(ctx, a_half), dai(ctx, a_int8), dbh(ctx, b_half);
    struct Row { const char *name, *kernel; const Dev *a, *b; int out; };   // out: 0 f32, 1 half, 2 i32
    const Row rows[] = {
        {"FP4 E2M1 g16 -> FP32 accumulate", "fp4_e2m1_matmul_benchmark", &dap, &dbp, 0},
        {"half x FP4 E2M1 g16 -> half accumulate", "half_fp4_matmul_half_benchmark", &dah, &dbp, 1},
        {"half x INT4 -> half accumulate", "half_int4_matmul_half_benchmark", &dah, &dbp, 1},
        {"INT8 x half -> half accumulate", "int8_half_matmul_half_benchmark", &dai, &dbh, 1},
        {"INT4 x INT4 -> INT32 accumulate", "int4_int8_matmul_benchmark", &dap, &dbp, 2},
    };
    const mpp41_matmul_config cfg = {M, N, K, K / 2};
    for (const Row &r : rows) {
        Dev c(ctx, (size_t)M * N * (r.out == 1 ? 2 : 4));
        Dev ws(ctx, mpp41_matmul_workspace_bytes(r.kernel, &cfg));
        check(mpp41_matmul(ctx, r.kernel, r.a->p, r.b->p, c.p, &cfg, ws.p), r.kernel);   // warm-up
        check(mpp41_synchronize(ctx), "synchronize");
        double t0 = 0, t1 = 0;
        {
            // time with the host clock around a synchronised batch (the C ABI
            // exposes only synchronize; the MLP rows use mpp41_mlp_benchmark)
            struct timespec a, b;
            clock_gettime(CLOCK_MONOTONIC, &a);
            for (int i = 0; i < g_iterations; ++i) check(mpp41_matmul(ctx, r.kernel, r.a->p, r.b->p, c.p, &cfg, ws.p), r.kernel);
            check(mpp41_synchronize(ctx), "synchronize");
            clock_gettime(CLOCK_MONOTONIC, &b);
            t0 = a.tv_sec + a.tv_nsec * 1e-9;
            t1 = b.tv_sec + b.tv_nsec * 1e-9;
        }
        const double sec = t1 - t0;
        const double tops = 2.0 * M * N * (double)K * g_iterations / sec / 1e12;
        std::string cks;
        if (r.out == 0) { const auto h = c.get<float>(); cks = float_checksum(h.data(), h.size()); }
        else if (r.out == 1) { const auto h = c.get<uint16_t>(); cks = half_raw_checksum(h.data(), h.size()); }
        else { const auto h = c.get<int32_t>(); cks = int_checksum(h.data(), h.size()); }
        printf("  %s:\n    %.3f ms/matmul, %.3f effective TOPS\n    checksum: %s\n", r.name,
               sec * 1e3 / g_iterations, tops, cks.c_str());
    }
}

// ---------------------------------------------------------------- MLP rows
void run_mlp(mpp41_ctx *ctx)
{
    const uint32_t T = 128, H = 1024, I = 4096;
    printf("\nGated MLP benchmark:\n  op: down(silu(gate(x)) * up(x))\n");
    printf("  shape: tokens=%u, hidden=%u, intermediate=%u\n  iterations: %d\n", T, H, I, g_iterations);
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
    for (const Row &r : rows) {
        mpp41_mlp_desc d;
        check(mpp41_mlp_describe(r.kernel, T, H, I, &d), r.kernel);
        const size_t out_elem = d.out_dtype == MPP41_F16 ? 2 : 4;
        Dev out(ctx, (size_t)T * H * out_elem), scratch(ctx, mpp41_mlp_scratch_bytes(&d));
        const void *x = d.afmt == MPP41_A_S8 ? x_int8.p : x_half.p;
        double sec = 0;
        check(mpp41_mlp_benchmark(ctx, &d, x, r.w->g.p, r.w->u.p, r.w->d.p, r.mx ? (const uint8_t *)sg.p : nullptr,
                                  r.mx ? (const uint8_t *)su.p : nullptr, r.mx ? (const uint8_t *)sd.p : nullptr,
                                  scratch.p, out.p, g_iterations, &sec),
              r.kernel);
        const double tops = 2.0 * 3.0 * T * (double)H * I * g_iterations / sec / 1e12;
        std::string cks;
        if (d.out_dtype == MPP41_S32) { const auto h = out.get<int32_t>(); cks = int_checksum(h.data(), h.size()); }
        else if (d.out_dtype == MPP41_F16) { const auto h = out.get<uint16_t>(); cks = half_raw_checksum(h.data(), h.size()); }
        else { const auto h = out.get<float>(); cks = float_checksum(h.data(), h.size()); }
        printf("  %s:\n    %.3f ms/MLP, %.3f effective TOPS\n    checksum: %s\n", r.name, sec * 1e3 / g_iterations,
               tops, cks.c_str());
    }
    delete halfw; delete i8w; delete i4w; delete i2w; delete f4w; delete e4w; delete e5w;
}

}  // namespace

int main(int argc, char **argv)
{
    bool bench = false, mlp = false, accum = false;
    for (int i = 1; i < argc; ++i) {
        if (!strcmp(argv[i], "--benchmark")) bench = true;
        else if (!strcmp(argv[i], "--mlp-benchmark")) mlp = true;
        else if (!strcmp(argv[i], "--accum-probe")) accum = true;
        else if (!strcmp(argv[i], "--skip-tensor")) {}
        else if (!strcmp(argv[i], "--iterations") && i + 1 < argc) g_iterations = atoi(argv[++i]);
        else { fprintf(stderr, "unknown argument %s\n", argv[i]); return 2; }
    }
    if (g_iterations < 1) g_iterations = 1;
    mpp41_ctx *ctx = nullptr;
    check(mpp41_create(0, &ctx), "mpp41_create");
    char name[256];
    check(mpp41_device_name(ctx, name, sizeof(name)), "device name");
    printf("Device: %s\n", name);
    const bool ok = run_roundtrips(ctx);
    printf("MTLTensor creation probe: not applicable (Metal host API).\n");
    if (bench) run_big_matmul(ctx);
    if (mlp) run_mlp(ctx);
    if (accum) printf("Accumulator precision probe: not applicable (Apple matmul2d semantics).\n");
    mpp41_destroy(ctx);
    if (!ok) {
        fprintf(stderr, "error: One or more packed numeric checks failed.\n");
        return 1;
    }
    printf("PASS\n");
    return 0;
}
