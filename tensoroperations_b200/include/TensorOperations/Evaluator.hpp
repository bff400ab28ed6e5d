// Evaluator.hpp -- policy tags (TeamPolicyTag, TeamPolicyTag2) and
// Evaluator<TeamPolicyTag, Node, Tile> (scratch sizing of the tree route).
#pragma once
#include <TensorOperations/b200/Graph.hpp>
#include <TensorOperations/Graph.hpp>
