// Drop-in include path: a host program written against the reference
// (`#include "model/ppo.h"`) compiles unchanged with -I<this include directory>.
#pragma once
#include "../metalgym/ppo.h"
