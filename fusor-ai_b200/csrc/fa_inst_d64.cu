// attend_kernel instantiations for head_dim 64.
#define FA_HEAD_DIM 64
#include "fa_inst.cuh"
