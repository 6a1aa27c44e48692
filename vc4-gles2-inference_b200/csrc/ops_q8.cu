// ops_q8.cu -- q8 matvec kernels (see ops_wt.inc).
#define VC4_WT W_Q8
#define VC4_SUF q8
#include "ops_wt.inc"
