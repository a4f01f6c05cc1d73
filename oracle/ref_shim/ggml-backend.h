/* Shim (TEST INFRASTRUCTURE ONLY): the two handle types imi/model.h names. The CPU_REPACK path is not used. */
#pragma once
#include "ggml.h"
typedef struct ggml_backend_buffer_type *ggml_backend_buffer_type_t;
typedef struct ggml_backend_buffer *ggml_backend_buffer_t;
