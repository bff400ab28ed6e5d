// NodeHandle.hpp -- node kinds and the make_*_node factories.
#pragma once
#include <TensorOperations/b200/Nodes.hpp>
