// The emulator's inline-PTX layer for the host build of the device kernels:
// named by L3G_PTX_HEADER in place of l3g_ptx.cuh and l3g_tcgen05.cuh
// (included inside namespace l3g).  Test infrastructure only.
#pragma once

#include "simt_ptx.h"

#include "simt_tcgen05_helpers.h"
