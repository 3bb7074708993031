/* See ggml.h in this folder: declarations-only stand-in, nothing defined. */
#pragma once
#include "ggml.h"
