// ops_q4.cu -- q4 matvec kernels (see ops_wt.inc).
#define VC4_WT W_Q4
#define VC4_SUF q4
#include "ops_wt.inc"
