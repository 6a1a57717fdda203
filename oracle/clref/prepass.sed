# Source pre-pass for compiling kernels/gemm.cl and kernels/conv_ov.cl as C++
# through ocl_shim.h (TEST INFRASTRUCTURE ONLY; the output goes to oracle/_ref/).
# OpenCL vector literals with one level of parentheses -> brace initialisers
s/(half2)(\([^()]*\))/half2{\1}/g
# vector components -> subscripts
s/\.s0\b/[0]/g
s/\.s1\b/[1]/g
# work-group arrays -> group-shared statics; `__local` elsewhere (pointer
# declarations and casts into those arrays) carries no meaning on the CPU
s/__local half As_\[/IVB_GROUP_ARRAY half As_[/
s/__local half Bs_\[/IVB_GROUP_ARRAY half Bs_[/
s/__local half2 partial\[/IVB_GROUP_ARRAY half2 partial[/
s/__local //g
