// kvb_api_atoms.cu - kvb_atom_read (include/kvb.h): validation and launch of TILT's moment-atom read
// (kvb_atoms.cuh).
#include <cuda_runtime.h>

#include "kvb_host.h"
#include "kvb_common.cuh"
#include "kvb_atoms.cuh"

extern "C" kvb_status kvb_atom_read(const kvb_atoms* m, const float* qs, int Hq, int c, float* logit, float* cfac,
                                    float* tB, void* stream) {
    if (!m || !qs || !logit || !cfac) return fail(KVB_EINVAL, "atom_read: null argument");
    if (m->B <= 0 || m->Hkv <= 0 || m->NA <= 0 || m->d <= 0 || m->d > kvb::AT_MAX_D || m->r < 1 ||
        m->r > kvb::AT_MAX_R || Hq <= 0 || Hq % m->Hkv || c <= 0 || (m->order != 1 && m->order != 2))
        return fail(KVB_EINVAL, "atom_read: shapes (d <= %d, 1 <= r <= %d, Hq a multiple of Hkv, order 1 or 2)",
                    kvb::AT_MAX_D, kvb::AT_MAX_R);
    if (!m->mu_k || !m->logn || (m->order == 2 && (!m->U || !m->lam || !m->diag || (m->project && !m->R))) ||
        (m->tilt && (!m->A || !m->Bk || !m->Rv || !tB)))
        return fail(KVB_EINVAL, "atom_read: a tensor the flags need is null");
    kvb::atom_read_kernel<<<unsigned(m->B * m->Hkv * m->NA), kvb::AT_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
        *m, qs, Hq, c, logit, cfac, tB);
    return launch_check("atom_read");
}

KVB_STATUS_WORDS(status_words_atoms)
