/* Stand-in for MAGMA's LAPACK header (see magma_v2.h in this folder). */
#pragma once
#include "magma_v2.h"
