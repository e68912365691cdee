// Semantic diversity pruning: the pair resolution of MentatGenerator._prune_similar
// (core/generator.py:400-497) on the device.
//
// The reference builds the similarity of a tree's warmed-up leaves with
// F.normalize + torch.mm (:441-444), masks the diagonal, the lower triangle and
// sibling pairs (:446-458), takes the pairs above the threshold with nonzero()
// (:463), reads them to the host with tolist() and resolves them in row-major
// order (:470-484): a pair whose leaves are both still unpruned prunes the one
// with the lower cumulative log-prob (the second on a tie).  This kernel takes
// the similarity matrix (the same torch call) and replaces the masking, the
// nonzero / tolist round trip and the host loop; the host reads one flag per
// leaf.
//
// One warp per tree.  Rows are resolved one after another (a row's outcome
// depends on every earlier row), each row 32 columns at a time with ballots:
// the candidates of a chunk are its columns above the threshold whose leaf is
// still unpruned; the first candidate that stops the row (its log-prob beats
// row i's, or it is i itself) prunes i, and every candidate before it is pruned.
// The masked entries are compared as sim x 0, as the reference's (sim * mask) >
// threshold does, so a negative threshold behaves as it does there.

#include "common.cuh"

namespace mentat {

constexpr int PRUNE_MAX = 4096;  // leaves of one tree

template <typename S>
__global__ void __launch_bounds__(32) k_prune_pairs(const S* __restrict__ sim, int64_t stride,
                                                    const int32_t* __restrict__ group_off, int ngroups,
                                                    const int64_t* __restrict__ parent_key,
                                                    const double* __restrict__ logp, float thr,
                                                    uint8_t* __restrict__ out) {
    __shared__ uint8_t pr[PRUNE_MAX];
    const int g = blockIdx.x;
    if (g >= ngroups) return;
    const int lane = threadIdx.x;
    const int a = group_off[g];
    const int M = min(group_off[g + 1] - a, PRUNE_MAX);
    for (int k = lane; k < M; k += 32) pr[k] = 0;
    __syncwarp();
    for (int i = 0; i < M; ++i) {
        if (pr[i]) continue;  // warp-uniform: read after the last __syncwarp
        const double lpi = logp[a + i];
        const int64_t pki = parent_key[a + i];
        const S* row = sim + (int64_t)(a + i) * stride + a;
        bool dead = false;
        for (int j0 = 0; j0 < M && !dead; j0 += 32) {
            const int j = j0 + lane;
            bool cand = false, stop = false;
            if (j < M) {
                const bool keep = j > i && pki != parent_key[a + j];  // upper triangle, not siblings
                float v = Elem<S>::to_f(row[j]);
                if (!keep) v *= 0.f;
                cand = v > thr && !pr[j];
                // Python's `lp_i >= lp_j` is False for NaN: the else branch prunes i
                stop = cand && (j == i || !(lpi >= logp[a + j]));
            }
            const unsigned cm = __ballot_sync(0xffffffffu, cand);
            const unsigned sm = __ballot_sync(0xffffffffu, stop);
            unsigned kill = cm;
            if (sm) {
                kill = cm & ((1u << (__ffs(sm) - 1)) - 1u);  // the candidates before the stop
                dead = true;
            }
            if ((kill >> lane) & 1u) pr[j] = 1;
            if (dead && lane == 0) pr[i] = 1;
            __syncwarp();
        }
    }
    for (int k = lane; k < M; k += 32) out[a + k] = pr[k];
}

}  // namespace mentat

using namespace mentat;

extern "C" int mentat_prune_similar(const void* sim, int32_t dtype, int64_t sim_stride, const int32_t* group_off,
                                    int32_t ngroups, int32_t max_group, const int64_t* parent_key,
                                    const double* logp, float threshold, uint8_t* prune_out, cudaStream_t s) {
    if (ngroups < 0 || max_group < 0 || max_group > PRUNE_MAX || sim_stride < 0) return MENTAT_ERR_ARG;
    if (ngroups == 0) return MENTAT_OK;
    if (!sim || !group_off || !parent_key || !logp || !prune_out) return MENTAT_ERR_ARG;
    switch (dtype) {
        case MENTAT_F32:
            k_prune_pairs<float><<<ngroups, 32, 0, s>>>(reinterpret_cast<const float*>(sim), sim_stride, group_off,
                                                        ngroups, parent_key, logp, threshold, prune_out);
            break;
        case MENTAT_BF16:
            k_prune_pairs<__nv_bfloat16><<<ngroups, 32, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(sim),
                                                                sim_stride, group_off, ngroups, parent_key, logp,
                                                                threshold, prune_out);
            break;
        case MENTAT_F16:
            k_prune_pairs<__half><<<ngroups, 32, 0, s>>>(reinterpret_cast<const __half*>(sim), sim_stride, group_off,
                                                         ngroups, parent_key, logp, threshold, prune_out);
            break;
        default: return MENTAT_ERR_UNSUPPORTED;
    }
    MENTAT_CHECK_LAUNCH();
    return MENTAT_OK;
}
