// The whole library as one translation unit (one definition of the device error word, no device linking).
#include "lb_quant.cu"
#include "lb_gemv.cu"
#include "lb_gemm.cu"
#include "lb_api.cu"
#include "lb_noalloc.cu"
#include "lb_peer.cu"
#include "lb_norm.cu"
#include "lb_act.cu"
