// attend_kernel instantiations for head_dim 128.
#define FA_HEAD_DIM 128
#include "fa_inst.cuh"
