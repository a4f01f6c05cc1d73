// Drop-in: imi's brain.h for callers compiled against the B200 engine (this directory first on the include path).
#pragma once
#include "../imi_brain_cuda.h"
