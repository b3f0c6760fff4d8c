// compat.h — force-included when the Genllm engine sources are compiled here
// (test infrastructure only): GCC 13's libstdc++ lacks C++23 <print>,
// std::formatter<std::vector> and std::expf, which those sources use.
#pragma once
#include <cmath>

#include "print"

namespace std {
using ::expf;
}
