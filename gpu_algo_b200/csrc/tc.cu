// placeholder until the tcgen05 engine lands
#include "common.cuh"
#include "internal.h"
namespace bfk {
bool tc_supported(int, int) { return false; }
bool tc_make_plan(int64_t, int64_t, int, int, int, int, TcPlan *) { return false; }
int tc_run(const float *, const float *, int64_t, float *, int32_t *, void *, const TcPlan &,
           cudaStream_t, cudaEvent_t, cudaEvent_t, int *) { return 1; }
const void *tc_kernel_ptr(int, int) { return nullptr; }
size_t tc_smem_bytes(int, int) { return 0; }
}
