// Drop-in: imi's model.h (the model file) for callers compiled against the B200 engine: imi_file over the library's
// own GGUF reader, with the gguf accessors the reference's callers use (this directory first on the include path).
#pragma once
#include "../imi_file_cuda.h"
