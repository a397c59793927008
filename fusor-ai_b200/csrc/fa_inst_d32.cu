// attend_kernel instantiations for head_dim 32.
#define FA_HEAD_DIM 32
#include "fa_inst.cuh"
