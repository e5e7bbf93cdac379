// Fused EXL3 projection: host dispatch over codebook and row count (kernels in sx_gemv_impl.cuh,
// instantiated per codebook in sx_gemv_{mcg,mul1,hash,pair1}.cu).
#include <mutex>
#include <utility>
#include <vector>

#include "sx_kernels.h"
#include "sx_decode.cuh"

namespace sx {

template <int KIND, int NB, bool W16>
cudaError_t dispatch_n(const GemvArgs& a, int n, int groups, cudaStream_t stream);

struct SplitKey {
    const void* kern;
    int out, in, groups, mg;
    bool operator==(const SplitKey& o) const {
        return kern == o.kern && out == o.out && in == o.in && groups == o.groups && mg == o.mg;
    }
};

namespace {
std::mutex g_split_lock;
std::vector<std::pair<SplitKey, int>> g_splits;
}  // namespace

int cached_split(const SplitKey& k) {
    std::lock_guard<std::mutex> guard(g_split_lock);
    for (const auto& e : g_splits)
        if (e.first == k) return e.second;
    return 0;
}

void remember_split(const SplitKey& k, int S) {
    std::lock_guard<std::mutex> guard(g_split_lock);
    g_splits.emplace_back(k, S);
}

cudaError_t launch_gemv(const GemvArgs& a, int kind, int n, int groups, cudaStream_t stream) {
    const int nb = (a.rows + 7) / 8;
    const bool w16 = a.wmask == 0xFFFFu;
#define SX_KIND(K)                                                                                   \
    case K:                                                                                          \
        if (nb == 1) return w16 ? dispatch_n<K, 1, true>(a, n, groups, stream) : dispatch_n<K, 1, false>(a, n, groups, stream); \
        return w16 ? dispatch_n<K, 2, true>(a, n, groups, stream) : dispatch_n<K, 2, false>(a, n, groups, stream);
    switch (kind) {
        SX_KIND(K_MUL1)
        SX_KIND(K_MCG)
        SX_KIND(K_HASH)
        case K_PAIR1:
            return nb == 1 ? dispatch_n<K_PAIR1, 1, true>(a, n, groups, stream)
                           : dispatch_n<K_PAIR1, 2, true>(a, n, groups, stream);
        default: return cudaErrorInvalidValue;
    }
#undef SX_KIND
}

}  // namespace sx
