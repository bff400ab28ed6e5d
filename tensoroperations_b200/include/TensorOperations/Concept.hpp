// Concept.hpp -- TensorLike and CombineLike.
#pragma once
#include <TensorOperations/b200/Nodes.hpp>
