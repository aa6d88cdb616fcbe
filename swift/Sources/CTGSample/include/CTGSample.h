/* Umbrella header of the CTGSample module: the engine's C ABI, unchanged. */
#ifndef CTGSAMPLE_H
#define CTGSAMPLE_H
#include "../../../../include/tgsample.h"
#endif
