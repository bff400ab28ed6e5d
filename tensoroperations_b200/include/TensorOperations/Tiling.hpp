// Tiling.hpp -- StaticTile<extents...>, Tile<A, B, C>, CombineTile<Out, Ops...>.
#pragma once
#include <TensorOperations/b200/Labels.hpp>
#include <TensorOperations/b200/TileSpec.hpp>
