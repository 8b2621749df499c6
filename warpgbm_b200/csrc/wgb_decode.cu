// Host-side tree decode of warpgbm_b200 (plain C++, no device code).
//
// Turns one tree of the engine's level-packed node records (what
// wgb_level_split / wgb_level_partition leave in ws->nodes) into the
// pre-order arrays that prediction and the reference's nested-dict trees
// are built from, and adds the tree's per-era split gains to the
// importance matrix in pre-order -- the order in which the reference's
// depth-first growth adds them (warpgbm/core.py:624-627).
#include "wgb_common.cuh"

namespace wgb {

struct TreeDecoder {
    const wgb_node *nodes;
    int D, ntree;
    const int32_t *feats;
    const float *gain;
    int E;
    float *imp;
    int F;
    int32_t *packed;
    float *leaf;
    int64_t *samples;
    int64_t cap, n = 0;
    bool bad = false;

    long long base(int d) const { return (long long)ntree * ((1ll << d) - 1); }

    void emit(int d, long long r) {
        if (bad) return;
        if (n >= cap || r < 0 || r >= ((long long)ntree << d)) {
            bad = true;
            return;
        }
        const long long g = base(d) + r;
        const wgb_node &nd = nodes[g];
        const int64_t id = n++;
        if (d < D && nd.fpos >= 0) {
            const int f = feats[nd.fpos];
            if (imp && f >= 0 && f < F)
                for (int e = 0; e < E; ++e) imp[(long long)e * F + f] += gain[g * E + e];
            packed[2 * id] = f;
            leaf[id] = 0.0f;
            samples[id] = 0;
            emit(d + 1, nd.child);
            const int64_t right = n;
            emit(d + 1, (long long)nd.child + 1);
            packed[2 * id + 1] = (int32_t)((nd.bin & 0xFF) | (right << 8));
        } else {
            int32_t bits;
            static_assert(sizeof(bits) == sizeof(nd.leaf), "leaf is 32-bit");
            __builtin_memcpy(&bits, &nd.leaf, sizeof(bits));
            packed[2 * id] = -1;
            packed[2 * id + 1] = bits;
            leaf[id] = nd.leaf;
            samples[id] = nd.count;
        }
    }
};

}  // namespace wgb

extern "C" int64_t wgb_decode_tree(const wgb_node *nodes, int32_t D, int32_t ntree, int32_t root,
                                   const int32_t *feats, const float *era_gain, int32_t E, float *imp,
                                   int32_t F, int32_t *packed, float *leaf, int64_t *samples, int64_t cap) {
    if (!nodes || !feats || !packed || !leaf || !samples || D < 1 || D > 24 || E < 1 ||
        (imp && (!era_gain || F < 1))) {
        wgb::set_error("wgb_decode_tree: bad arguments");
        return -WGB_ERR_ARG;
    }
    const int nt = ntree > 1 ? ntree : 1;
    if (root < 0 || root >= nt) {
        wgb::set_error("wgb_decode_tree: root %d out of range", root);
        return -WGB_ERR_ARG;
    }
    wgb::TreeDecoder dec{nodes, D, nt, feats, era_gain, E, imp, F, packed, leaf, samples, cap};
    dec.emit(0, root);
    if (dec.bad) {
        wgb::set_error("wgb_decode_tree: malformed records or output too small (cap %lld)", (long long)cap);
        return -WGB_ERR_ARG;
    }
    return dec.n;
}
