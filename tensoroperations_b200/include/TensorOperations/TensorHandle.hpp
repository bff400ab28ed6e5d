// TensorHandle.hpp -- make_handle<labels...>(view).
#pragma once
#include <TensorOperations/b200/Nodes.hpp>
