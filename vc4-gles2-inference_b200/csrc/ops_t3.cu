// ops_t3.cu -- t3 matvec kernels (see ops_wt.inc).
#define VC4_WT W_T3
#define VC4_SUF t3
#include "ops_wt.inc"
