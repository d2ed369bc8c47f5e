// Host-only check of the decode kernel's stream-K partitions (gptoss-infer_b200/csrc/streamk.cuh), built and run by
// tests/test_streamk_cpu.py; no GPU is used. For several shapes and grid sizes, both parts (gate/up split by equal
// units, down by the cost model), it checks that:
//   * the CTA ranges are contiguous, start at 0, end at the part's total and are cut only at stage starts;
//   * the stages of all CTAs cover every unit of the part exactly once, none longer than 4 units or crossing a slot;
//   * every tile has exactly one finalizer (the CTA holding its first unit, whose segment of it is its last) and at
//     most kMaxContrib contributors, so it fits the partial-sum slots;
//   * the 20b shape's gate/up split is the plain equal-unit split the kernel was measured with.
// Prints one line per failure and exits with status 1 if any.
#include <cstdio>
#include <vector>

#include "../gptoss-infer_b200/csrc/streamk.cuh"

using namespace gpt::sk;

static int failures = 0;
#define CHECK(cond, ...)                       \
    do {                                       \
        if (!(cond)) {                         \
            ++failures;                        \
            std::printf("FAIL: " __VA_ARGS__); \
            std::printf("\n");                 \
        }                                      \
    } while (0)

static void parts(int k, int H, int I, Part& g, Part& d) {
    constexpr int TR = 256;                   // kDecodeTileRows
    g = Part{};
    g.mode = kGateUp;
    g.RT = (2 * I + TR - 1) / TR;
    g.n_tiles = k * g.RT;
    g.UK = H / 64;
    g.UT = g.UK;
    g.total = (long long)g.n_tiles * g.UT;
    d = Part{};
    d.mode = kDown;
    d.RT = (H + TR - 1) / TR;
    d.n_tiles = d.RT;
    d.UK = I / 64;
    d.UT = k * d.UK;
    d.total = (long long)d.n_tiles * d.UT;
}

static bool is_stage_start(const Part& p, long long u) {
    if (u == p.total) return true;
    const long long t = u / p.UT;
    const int m = int(u - t * p.UT);
    const int ku = p.mode == kGateUp ? m : m % p.UK;
    return ku % 4 == 0;
}

static void check_part(const char* name, const Part& p, const std::vector<long long>& B, int nc, int k, int H, int I) {
    CHECK(int(B.size()) == nc + 1 && B[0] == 0 && B[nc] == p.total, "%s k=%d H=%d I=%d nc=%d: bounds ends", name, k,
          H, I, nc);
    for (int c = 0; c < nc; ++c) {
        CHECK(B[c] <= B[c + 1], "%s k=%d H=%d I=%d nc=%d: bounds decrease at %d", name, k, H, I, nc, c);
        CHECK(is_stage_start(p, B[c]), "%s k=%d H=%d I=%d nc=%d: cut inside a stage at CTA %d", name, k, H, I, nc, c);
    }
    std::vector<int> covered(size_t(p.total), 0);
    std::vector<int> finalizers(size_t(p.n_tiles), 0);
    for (int c = 0; c < nc; ++c) {
        const int n = build_stages(p, B.data(), c, nullptr, 0, 0, 0, nullptr);
        std::vector<Stage> st(size_t(n > 0 ? n : 1));
        build_stages(p, B.data(), c, st.data(), 0, n, 0, nullptr);
        fill_tile_info(p, B.data(), nc, c, st.data(), 0, n);
        for (int i = 0; i < n; ++i) {
            const Stage& s = st[size_t(i)];
            CHECK(s.nu >= 1 && s.nu <= 4 && s.ku0 % 4 == 0 && s.ku0 + s.nu <= p.UK,
                  "%s k=%d H=%d I=%d nc=%d: bad stage (ku0 %d, nu %d)", name, k, H, I, nc, s.ku0, s.nu);
            const long long base = (long long)s.tile * p.UT + (p.mode == kGateUp ? 0 : (long long)s.s * p.UK);
            for (int u = 0; u < s.nu; ++u) {
                const long long unit = base + s.ku0 + u;
                if (unit >= 0 && unit < p.total) ++covered[size_t(unit)];
            }
            if (s.last) {
                CHECK(s.whole >= 0, "%s k=%d H=%d I=%d nc=%d: tile %d over the partial-sum slots", name, k, H, I, nc,
                      s.tile);
                if (s.whole == 1 || c == s.cf) ++finalizers[size_t(s.tile)];
            }
        }
    }
    long long bad = 0;
    for (int v : covered) bad += v != 1;
    CHECK(bad == 0, "%s k=%d H=%d I=%d nc=%d: %lld units not covered exactly once", name, k, H, I, nc, bad);
    for (int t = 0; t < p.n_tiles; ++t) {
        int cf = 0, cl = 0;
        tile_contributors(p, B.data(), nc, t, cf, cl);
        CHECK(cl - cf + 1 <= kMaxContrib, "%s k=%d H=%d I=%d nc=%d: tile %d spans %d CTAs", name, k, H, I, nc, t,
              cl - cf + 1);
        CHECK(finalizers[size_t(t)] == 1, "%s k=%d H=%d I=%d nc=%d: tile %d has %d finalizers", name, k, H, I, nc, t,
              finalizers[size_t(t)]);
    }
}

int main() {
    const int shapes[][3] = {{4, 2880, 2880}, {2, 512, 256}, {1, 64, 64}, {8, 1024, 1024}, {4, 2880, 1408},
                             {8, 2880, 2880}, {4, 4096, 2048}};
    const int grids[] = {148, 132, 160};
    for (const auto& sh : shapes)
        for (int nc : grids) {
            Part g, d;
            parts(sh[0], sh[1], sh[2], g, d);
            check_part("gate/up", g, equal_bounds(g, nc), nc, sh[0], sh[1], sh[2]);
            check_part("down", d, balanced_bounds(d, nc, kDownCost), nc, sh[0], sh[1], sh[2]);
        }
    // the 20b shape's gate/up split on 148 SMs: unit c * total / nc rounded up to the next stage start
    Part g, d;
    parts(4, 2880, 2880, g, d);
    const std::vector<long long> B = equal_bounds(g, 148);
    for (int c = 0; c <= 148; ++c) {
        const long long u = (long long)c * g.total / 148, t = u / g.UT;
        const int m = int(u - t * g.UT), ku2 = (m + 3) & ~3;
        const long long want = t * g.UT + (ku2 < g.UK ? ku2 : g.UK);
        CHECK(B[size_t(c)] == want, "20b gate/up split differs at CTA %d", c);
    }
    if (failures == 0) std::printf("OK\n");
    return failures ? 1 : 0;
}
