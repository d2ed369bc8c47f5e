// Stream-K work partition of the tensor-core MoE GEMVs, shared by host (shared-memory sizing) and device.
//
// The MMA unit is K = 64 of one tile of weight rows (256 in the decode kernel). A GEMV "part" is n_tiles tiles of UT
// units each (gate/up: a tile is rows of one selected expert and UT = UK units of K; down: a tile is output rows and
// UT = k * UK units, the k experts' rows laid end to end). CTA c of nc takes the contiguous units [B(c), B(c+1)),
// cut at stage starts (a stage is at most 4 units, one 128-byte-wide TMA box of K, within one slot); the cuts
// balance a per-CTA cost (stages, segments, tiles finalized) rather than the unit count, because every tile ends in
// a short stage and finalizing a tile costs about as much as three stages. A tile split between CTAs is finished by
// its first contributor (for which the tile is its last segment), which adds the others' partial sums in CTA order.
#pragma once
#include <cstdint>
#include <vector>

namespace gpt {
namespace sk {

constexpr int kMaxContrib = 16;                // CTAs that may share one tile

enum Mode { kGateUp = 0, kDown = 1 };

struct Part {
    int mode;
    int n_tiles;        // gate/up: k * RT; down: RT
    int RT;             // 128-row tiles per expert matrix
    int UK;             // MMA units (K = 64) per slot
    int KT;             // scale chunks (K = 128) per row
    int SPS;            // stages (K = 256) per slot
    int UT;             // units per tile
    long long total;    // n_tiles * UT
    unsigned long long* partial;   // [n_tiles][kMaxContrib][rows]: (launch epoch << 32) | fp32 bits of a partial sum
};

struct Stage {
    int tile;
    short s, ku0, nu;   // slot, first unit in the slot, units in this stage (1..4)
    short first, last;  // first / last stage of this CTA's segment of the tile
    short seg;          // segment index within this CTA (both parts counted together)
    short mode;         // kGateUp or kDown
    // filled on a segment's last stage (by fill_tile_info):
    short cf;           // first CTA sharing the tile; partial sums are stored at slot (cta - cf)
    short units;        // units of the tile this CTA computes
    short whole;        // 1: this CTA computes the whole tile
    unsigned short mask;  // bit i: CTA cf + i computes part of the tile
};

// Units of the stage that starts at unit u (stages are at most 4 units and never cross a slot).
inline int stage_units_at(const Part& p, long long u) {
    const long long t = u / p.UT;
    const int m = int(u - t * p.UT);
    const int ku = p.mode == kGateUp ? m : m % p.UK;
    const int left = p.UK - ku;
    return left < 4 ? left : 4;
}

// Cost model of a CTA's range (cycles on a B200, from the kernel's clock64 trace): each stage a fixed issue cost plus
// a cost per unit, each segment (the part of one tile in the range) an accumulator drain and publication, and each
// tile whose first unit lies in the range its finalization (the range's CTA is the tile's first contributor).
struct CostModel {
    double stage, unit, segment, finalize;
};

// The decode kernel's down part, from its clock64 trace on a B200: a stage ≈ 500 + 145 per unit (1.08K for 4 units,
// the weights already resident), a segment's drain and publication ≈ 1.5K, finalizing a tile (partial sums,
// residual) ≈ 1.5K.
constexpr CostModel kDownCost{500.0, 145.0, 1500.0, 1500.0};

// Range boundaries of nc CTAs with equal unit counts: unit c * total / nc rounded up to the next stage start. A part
// of at most nc stages gets one stage per CTA for its first CTAs instead, so that no empty range falls between two
// CTAs sharing a tile (the partial-sum slots of a tile are indexed by CTA distance).
inline std::vector<long long> equal_bounds(const Part& p, int nc) {
    std::vector<long long> starts;
    for (long long u = 0; u < p.total && long(starts.size()) <= nc; u += stage_units_at(p, u)) starts.push_back(u);
    if (long(starts.size()) <= nc) {
        std::vector<long long> B(size_t(nc) + 1, p.total);
        for (size_t i = 0; i < starts.size(); ++i) B[i] = starts[i];
        return B;
    }
    std::vector<long long> B(size_t(nc) + 1);
    for (int c = 0; c <= nc; ++c) {
        const long long u = (long long)c * p.total / nc, t = u / p.UT;
        const int m = int(u - t * p.UT), s = m / p.UK, ku = m - s * p.UK, ku2 = (ku + 3) & ~3;
        B[c] = t * p.UT + (long long)s * p.UK + (ku2 < p.UK ? ku2 : p.UK);
    }
    return B;
}

// Range boundaries [B(0) = 0, ..., B(nc) = total] of the nc CTAs, cut only at stage starts, chosen so that the
// largest range cost is as small as possible (binary search over the cost bound, greedy filling); trailing CTAs may
// get empty ranges.
inline std::vector<long long> balanced_bounds(const Part& p, int nc, const CostModel& cm) {
    std::vector<long long> start;                  // unit of every stage start, then total
    std::vector<double> cost;                      // the stage's own cost
    std::vector<char> tile_first;                  // the stage starts a tile
    for (long long u = 0; u < p.total;) {
        const int nu = stage_units_at(p, u);
        start.push_back(u);
        cost.push_back(cm.stage + cm.unit * nu);
        tile_first.push_back(u % p.UT == 0);
        u += nu;
    }
    const size_t ns = start.size();
    start.push_back(p.total);
    // greedy: each range takes stages while its cost stays within X; returns the number of ranges, or nc + 1 when a
    // tile would be shared by more than kMaxContrib ranges (it has that many partial-sum slots)
    auto fill = [&](double X, std::vector<long long>* out) {
        int n = 0;
        size_t i = 0;
        long long last_tile = -1;
        int ranges_on_tile = 0;
        if (out) out->assign(1, 0);
        while (i < ns) {
            double c = 0.0;
            long long tile = -1;
            size_t j = i;
            while (j < ns) {
                const long long t = start[j] / p.UT;
                double add = cost[j] + (t != tile ? cm.segment : 0.0) + (tile_first[j] ? cm.finalize : 0.0);
                if (j > i && c + add > X) break;
                c += add;
                tile = t;
                ++j;
            }
            ++n;
            if (out) out->push_back(start[j]);
            const long long t0 = start[i] / p.UT, t1 = (start[j] - 1) / p.UT;   // tiles the range touches
            ranges_on_tile = t0 == last_tile ? ranges_on_tile + 1 : 1;
            if (ranges_on_tile > kMaxContrib) return nc + 1;
            if (t1 != t0) ranges_on_tile = 1;
            last_tile = t1;
            i = j;
        }
        return n;
    };
    double lo = 0.0, hi = 0.0;
    for (size_t i = 0; i < ns; ++i) hi += cost[i] + cm.segment + cm.finalize;
    for (int it = 0; it < 60; ++it) {
        const double mid = 0.5 * (lo + hi);
        if (fill(mid, nullptr) <= nc) hi = mid;
        else lo = mid;
    }
    std::vector<long long> B;
    fill(hi, &B);
    while (int(B.size()) < nc + 1) B.push_back(p.total);
    return B;
}

// Appends CTA c's stages of part p (range [B[c], B[c + 1])) to out[n0..] (at most cap entries in total); returns
// the new count. Segments are numbered from seg0.
inline int build_stages(const Part& p, const long long* B, int c, Stage* out, int n0, int cap, int seg0,
                        int* seg_end) {
    const long long B0 = B[c], B1 = B[c + 1];
    int n = n0, seg = seg0;
    for (long long u = B0; u < B1;) {
        const int t = int(u / p.UT);
        const long long Tend = (long long)(t + 1) * p.UT;
        const long long e = B1 < Tend ? B1 : Tend;
        int m = int(u - (long long)t * p.UT);
        const int m_end = int(e - (long long)t * p.UT);
        const int first_idx = n;
        while (m < m_end) {
            const int s = p.mode == kGateUp ? t / p.RT : m / p.UK;
            const int ku = p.mode == kGateUp ? m : m - s * p.UK;
            int nu = p.UK - ku < m_end - m ? p.UK - ku : m_end - m;
            nu = nu < 4 ? nu : 4;
            if (out && n < cap)
                out[n] = Stage{t, short(s), short(ku), short(nu), short(n == first_idx), 0, short(seg), short(p.mode),
                               0, 0, 0, 0};
            m += nu;
            ++n;
        }
        if (out && n > first_idx && n - 1 < cap) out[n - 1].last = 1;
        ++seg;
        u = e;
    }
    if (seg_end) *seg_end = seg;
    return n;
}

// CTAs whose ranges intersect tile t: [c_first, c_last] (the CTAs holding its first and last unit).
inline void tile_contributors(const Part& p, const long long* B, int nc, int t, int& c_first, int& c_last) {
    const long long T0 = (long long)t * p.UT, T1 = T0 + p.UT;
    auto owner = [&](long long u) {                  // the CTA whose (non-empty) range holds unit u
        int lo = 0, hi = nc - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) / 2;
            if (B[mid] <= u) lo = mid;
            else hi = mid - 1;
        }
        return lo;
    };
    c_first = owner(T0);
    c_last = owner(T1 - 1);
}

// Completes the segment-end entries of a stage list with who shares each tile.
inline void fill_tile_info(const Part& p, const long long* B, int nc, int c, Stage* st, int n0, int n1) {
    for (int i = n0; i < n1; ++i) {
        if (!st[i].last) continue;
        const int t = st[i].tile;
        const long long T0 = (long long)t * p.UT, T1 = T0 + p.UT;
        long long a = B[c], b = B[c + 1];
        a = a > T0 ? a : T0;
        b = b < T1 ? b : T1;
        st[i].units = short(b - a);
        st[i].whole = short(b - a == p.UT);
        int cf, cl;
        tile_contributors(p, B, nc, t, cf, cl);
        st[i].cf = short(cf);
        unsigned m = 0;
        for (int cc = cf; cc <= cl && cc - cf < kMaxContrib; ++cc) {
            long long x0 = B[cc], x1 = B[cc + 1];
            x0 = x0 > T0 ? x0 : T0;
            x1 = x1 < T1 ? x1 : T1;
            if (x0 < x1) m |= 1u << (cc - cf);
        }
        st[i].mask = (unsigned short)(cl - cf < kMaxContrib ? m : 0xFFFFu);   // 0xFFFF with cl-cf >= 16: error
        if (cl - cf >= kMaxContrib) st[i].whole = -1;
    }
}

__host__ __device__ __forceinline__ int nkt_of(const Stage& st) { return (st.ku0 + st.nu - 1) / 2 - st.ku0 / 2 + 1; }

// Runs of consecutive stage entries [a, b) whose scale chunks (and B stages) are contiguous both in global memory
// and in the per-entry shared regions (entry i owns 1 KB of scale chunks and one B stage).
template <class F>
__device__ __forceinline__ void for_each_run(const Stage* st, int n0, int n1, F&& f) {
    int a = n0;
    while (a < n1) {
        int b = a + 1;
        while (b < n1 && st[b - 1].mode == st[b].mode && st[b - 1].s == st[b].s && st[b - 1].tile == st[b].tile &&
               nkt_of(st[b - 1]) == 2 && st[b].ku0 == st[b - 1].ku0 + 4)
            ++b;
        int chunks = 0;
        for (int i = a; i < b; ++i) chunks += nkt_of(st[i]);
        f(a, b, chunks);
        a = b;
    }
}

}  // namespace sk
}  // namespace gpt
