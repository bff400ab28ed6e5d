// Graph.hpp -- make_graph / Graph::ops / Graph::execute (the tree route) and
// Evaluator<TeamPolicyTag, Node, Tile>::scratch_size_per_team.
#pragma once
#include <TensorOperations/DagGraph.hpp>
#include <TensorOperations/b200/Tree.hpp>
