// dense_chunk_tc.cu -- chunkwise (WY/UT) dense recurrence on tcgen05 tensor cores.
#include "dg_common.cuh"

namespace dg_host {

bool dense_chunked_tc_supports(int dtype, int B, int H, int T, int S, int Dh) {
    (void)dtype; (void)B; (void)H; (void)T; (void)S; (void)Dh;
    return false;
}

int dense_forward_chunked_tc(int, int, int, int, int, int, const void*, const void*, const void*,
                             const void*, const void*, int, const void*, void*, void*, float*,
                             float*, cudaStream_t) {
    return DG_ERR_UNSUPPORTED;
}

}  // namespace dg_host
