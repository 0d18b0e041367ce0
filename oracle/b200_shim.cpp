// Test infrastructure: the translation unit that gives the reference's apps their CUDA backend from
// libvarda_b200 through include/varda_b200_backend.hpp (see oracle/Makefile, target b200apps).
#define VARDA_B200_IMPLEMENT
#include "varda_b200_backend.hpp"
