// Drop-in: imi's core/seoul.h for callers compiled against the B200 engine (put this directory first on the include
// path; link libimi_cuda.so). The same class and calls as the reference's header, on the engine.
#pragma once
#include "../imi_seoul_cuda.h"
