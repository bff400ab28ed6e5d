// Evaluator.hpp -- policy tags (TeamPolicyTag, TeamPolicyTag2) and the evaluator entry.
#pragma once
#include <TensorOperations/b200/Graph.hpp>
