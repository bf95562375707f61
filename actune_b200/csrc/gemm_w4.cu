// Launchers of the group-64 tcgen05 GEMM for W = 4 (all A, all tile widths).
#include "gemm_launch.cuh"

ACTUNE_INSTANTIATE_GEMM(4)
