// DeviceTuple.hpp -- a heterogeneous tuple usable in device code.
#pragma once
#include <TensorOperations/b200/Nodes.hpp>
