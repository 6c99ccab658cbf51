// m4b_lib.cu -- single translation unit of libm4b.so.  The kernels share device symbols (the
// status word the bounded waits raise), so they are compiled together instead of with
// relocatable device code.
#include "m4b_kqkv.cu"
#include "m4b_gemv.cu"
#include "m4b_q8.cu"
#include "m4b_api.cu"
#include "m4b_noalloc.cu"
#include "m4b_exchange.cu"
