// Tiling.hpp -- StaticTile<extents...>.
#pragma once
#include <TensorOperations/b200/Labels.hpp>
