// Single translation unit of libwanflash: the device error word and wait
// limit are shared by every kernel, so the library is compiled as one unit
// (no relocatable device code or device link step needed).
#include "wf_capi.cu"
#include "wf_fwd.cu"
#include "wf_fwd2.cu"
#include "wf_bwd.cu"
#include "wf_bwd2.cu"
#include "wf_aux.cu"
#include "wf_noalloc.cu"
