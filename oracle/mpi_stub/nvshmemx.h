/* nvshmemx.h — see nvshmem.h beside it (TEST INFRASTRUCTURE ONLY). */
#include "nvshmem.h"
