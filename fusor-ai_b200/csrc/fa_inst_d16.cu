// attend_kernel instantiations for head_dim 16.
#define FA_HEAD_DIM 16
#include "fa_inst.cuh"
