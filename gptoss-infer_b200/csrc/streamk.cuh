// Stream-K work partition of the tensor-core MoE GEMVs, shared by host (shared-memory sizing) and device.
//
// The MMA unit is K = 64 of one tile of weight rows (256 in the decode kernel). A GEMV "part" is n_tiles tiles of UT
// units each (gate/up: a tile is rows of one selected expert and UT = UK units of K; down: a tile is output rows and
// UT = k * UK units, the k experts' rows laid end to end). CTA c of nc takes units [begin(c), begin(c+1)), begin
// rounded up to a 4-unit stage (one 128-byte-wide TMA box of K) within its slot, so every CTA streams about the same
// bytes. A tile split between CTAs is finished by its first contributor (for which the tile is its last segment),
// which adds the others' partial sums in CTA order.
#pragma once
#include <cstdint>

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

__host__ __device__ __forceinline__ long long stage_round(const Part& p, long long u) {
    const long long t = u / p.UT;
    const int m = int(u - t * p.UT);
    const int s = m / p.UK, ku = m - s * p.UK;
    const int ku2 = (ku + 3) & ~3;
    return t * p.UT + (long long)s * p.UK + (ku2 < p.UK ? ku2 : p.UK);
}

__host__ __device__ __forceinline__ long long cta_begin(const Part& p, int c, int nc) {
    return stage_round(p, (long long)c * p.total / nc);
}

// Appends CTA c's stages of part p to out[n0..] (at most cap entries in total); returns the new count. Segments are
// numbered from seg0.
__host__ __device__ inline int build_stages(const Part& p, int c, int nc, Stage* out, int n0, int cap, int seg0,
                                            int* seg_end) {
    const long long B0 = cta_begin(p, c, nc), B1 = cta_begin(p, c + 1, nc);
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

// CTAs whose ranges intersect tile t: [c_first, c_last].
__host__ __device__ inline void tile_contributors(const Part& p, int t, int nc, int& c_first, int& c_last) {
    const long long T0 = (long long)t * p.UT, T1 = T0 + p.UT;
    int c = int(T0 * nc / p.total);
    c = c < 0 ? 0 : (c > nc - 1 ? nc - 1 : c);
    while (c > 0 && cta_begin(p, c, nc) > T0) --c;
    while (c + 1 < nc && cta_begin(p, c + 1, nc) <= T0) ++c;
    c_first = c;
    int d = int((T1 - 1) * nc / p.total);
    d = d < c_first ? c_first : (d > nc - 1 ? nc - 1 : d);
    while (d > c_first && cta_begin(p, d, nc) > T1 - 1) --d;
    while (d + 1 < nc && cta_begin(p, d + 1, nc) <= T1 - 1) ++d;
    c_last = d;
}

// Completes the segment-end entries of a stage list with who shares each tile.
inline void fill_tile_info(const Part& p, int c, int nc, Stage* st, int n0, int n1) {
    for (int i = n0; i < n1; ++i) {
        if (!st[i].last) continue;
        const int t = st[i].tile;
        const long long T0 = (long long)t * p.UT, T1 = T0 + p.UT;
        long long a = cta_begin(p, c, nc), b = cta_begin(p, c + 1, nc);
        a = a > T0 ? a : T0;
        b = b < T1 ? b : T1;
        st[i].units = short(b - a);
        st[i].whole = short(b - a == p.UT);
        int cf, cl;
        tile_contributors(p, t, nc, cf, cl);
        st[i].cf = short(cf);
        unsigned m = 0;
        for (int cc = cf; cc <= cl && cc - cf < kMaxContrib; ++cc) {
            long long x0 = cta_begin(p, cc, nc), x1 = cta_begin(p, cc + 1, nc);
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
