// LevelPlan.hpp -- LevelPlan<levels>: slot counts and the three level guards.
#pragma once
#include <TensorOperations/b200/Plan.hpp>
