// Host-side check of the persistent decode kernel's work geometry
// (xl_kernels.h), for every weight width and grid it may meet:
//  * boxes: k-tiles of persist_tile_w(K) floats dividing K, at most 512 floats
//    per box, persist_boxes_per_group(K) boxes covering [0, K) exactly once;
//  * split projections (out-projection, W2): CTA b of G takes boxes
//    [b*T/G, (b+1)*T/G); the slot persist_contrib_slot gives each group's
//    contributing CTAs must be distinct, below persist_group_contrib, cover
//    every slot the staging sums (no slot left unwritten, which would be read
//    stale) and rise with the CTA index (the summation order);
//  * persist_max_contrib is the largest per-group count;
//  * the full model fits the kernel at every tensor-parallel width.
// Prints "ok" and exits 0, or prints the first failure and exits 1.
#include <cstdio>
#include <vector>

#include "xl_kernels.h"

using namespace xl;

static int fail(const char* what, int M, int K, int G, int g) {
    std::printf("FAIL %s: M=%d K=%d G=%d group=%d\n", what, M, K, G, g);
    return 1;
}

static int check_boxes(int K) {
    const int tw = persist_tile_w(K), kd = persist_box_tiles(K), bw = persist_box_width(K);
    const int nb = persist_boxes_per_group(K);
    if (K % tw || tw > 256 || kd < 1 || kd > K / tw || bw != tw * kd || bw > kPersistBoxK)
        return fail("box shape", 0, K, 0, -1);
    std::vector<int> hit(K, 0);
    for (int bi = 0; bi < nb; ++bi) {
        const int k0 = bi * bw;
        if (k0 >= K) return fail("box past K", 0, K, 0, bi);
        const int kc = K - k0 < bw ? K - k0 : bw;
        for (int k = k0; k < k0 + kc; ++k) ++hit[k];
    }
    for (int k = 0; k < K; ++k)
        if (hit[k] != 1) return fail("box coverage", 0, K, 0, k);
    return 0;
}

static int check_slots(int M, int K, int G) {
    const int nb = persist_boxes_per_group(K), groups = M / kPersistTileRows, T = groups * nb;
    std::vector<std::vector<int>> owner(groups);
    for (int g = 0; g < groups; ++g) owner[g].assign(persist_group_contrib(g, nb, T, G), -1);
    for (int b = 0; b < G; ++b) {
        const int t0 = b * T / G, t1 = (b + 1) * T / G;
        for (int tau = t0; tau < t1;) {
            const int g = tau / nb, bi0 = tau % nb, bi1 = nb < bi0 + (t1 - tau) ? nb : bi0 + (t1 - tau);
            const int c = persist_contrib_slot(b, g, bi0, nb, T, G);
            if (c < 0 || c >= static_cast<int>(owner[g].size())) return fail("slot out of range", M, K, G, g);
            if (owner[g][c] != -1) return fail("slot written twice", M, K, G, g);
            owner[g][c] = b;
            tau += bi1 - bi0;
        }
    }
    int mc = 0;
    for (int g = 0; g < groups; ++g) {
        const int n = static_cast<int>(owner[g].size());
        mc = n > mc ? n : mc;
        for (int c = 0; c < n; ++c) {
            if (owner[g][c] < 0) return fail("slot never written", M, K, G, g);
            if (c > 0 && owner[g][c] <= owner[g][c - 1]) return fail("slots out of CTA order", M, K, G, g);
        }
    }
    if (persist_max_contrib(M, K, G) != mc) return fail("persist_max_contrib", M, K, G, -1);
    return 0;
}

// XingLing-0.68B (hidden 1536, 24 heads, ffn 4096, context 768) on 148 SMs
// takes the persistent kernel at TP 1, 2, 4 and 8: shard widths are multiples
// of 64, each row group of the split projections has at most
// kPersistMaxContrib contributors, and the attention items fit the grid.
static int check_model_fits() {
    const int H = 1536, heads = 24, F = 4096, ctx = 768, G = 148;
    for (int tp : {1, 2, 4, 8}) {
        const int Hl = H / tp, Fl = F / tp, hl = heads / tp;
        if (Hl % kPersistKAlign || Fl % kPersistKAlign) return fail("shard width", H, Hl, tp, -1);
        if (persist_max_contrib(H, Hl, G) > kPersistMaxContrib) return fail("out-proj contributors", H, Hl, tp, -1);
        if (persist_max_contrib(H, Fl, G) > kPersistMaxContrib) return fail("W2 contributors", H, Fl, tp, -1);
        if (hl * persist_attn_ctas_per_head(ctx) > G) return fail("attention items", H, hl, tp, -1);
    }
    return 0;
}

int main() {
    int rc = check_model_fits();
    for (int K = kPersistKAlign; K <= 4096 && !rc; K += kPersistKAlign) rc = check_boxes(K);
    const int Ms[] = {256, 384, 640, 1024, 1536, 2048, 4096};
    const int Gs[] = {148, 132, 80, 8};
    for (int M : Ms)
        for (int K = kPersistKAlign; K <= 4096 && !rc; K += kPersistKAlign)
            for (int G : Gs)
                if (!rc) rc = check_slots(M, K, G);
    if (!rc) std::printf("ok\n");
    return rc;
}
