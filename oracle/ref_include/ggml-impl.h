// See ggml.h in this directory: nothing of this header is used by the hook.
#pragma once
#include "ggml.h"
