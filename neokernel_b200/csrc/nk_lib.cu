// Single translation unit of libnkgemm.so. The kernel families share device state (the
// bounded-wait error word nk::g_error), so they are compiled together rather than linked
// with relocatable device code.
#include "nk_gemv.cu"
#include "nk_tc.cu"
#include "nk_abi.cu"
#include "nk_static.cu"
#include "nk_decode.cu"
#include "nk_comm.cu"
