// LevelGraph.hpp -- make_level_graph / LevelGraph / LevelOutputs (B200 frontend).
#pragma once
#include <TensorOperations/LabelTiles.hpp>
#include <TensorOperations/LevelPlan.hpp>
#include <TensorOperations/b200/Graph.hpp>
