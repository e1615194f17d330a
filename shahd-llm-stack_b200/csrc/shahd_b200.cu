// The single translation unit of libshahd_b200.so: one device module, so the kernels share one
// g_shahd_device_error flag and one set of template instantiations.
#include "seam.cuh"
#include "session.cuh"
