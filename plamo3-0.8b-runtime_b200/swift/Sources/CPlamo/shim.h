/* The C ABI of libplamo_cuda as one Clang module for Swift: the runtime and batch entry points
 * (plamo.h) and the kernel-level ones (plamo_kernels.h), from the repository's include/. */
#include "../../../../include/plamo.h"
#include "../../../../include/plamo_kernels.h"
