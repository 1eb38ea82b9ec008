// TEST INFRASTRUCTURE ONLY: the reference's gym.h includes this metal-cpp
// header but uses nothing from it (see Foundation/Foundation.hpp).
#pragma once
