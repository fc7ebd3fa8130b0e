/* Empty stand-in: include/dit_manual.h includes ggml-cpu.h but uses nothing from it. */
#pragma once
#include "ggml.h"
