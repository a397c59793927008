// attend_kernel instantiations for head_dim 256.
#define FA_HEAD_DIM 256
#include "fa_inst.cuh"
