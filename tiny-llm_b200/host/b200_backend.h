// b200_backend.h — the GPU IBackend of libtqb200.so for the reference's QwenModel.
//
// create_b200_backend() returns an IBackend (runtime/backend.h:73-392) whose every op
// runs on the GPU through libtqb200.so (defined in b200_variants.cpp).  Pass it to
// QwenModel::create (runtime/qwen_model.h:117-122) as main.cpp does with
// create_cuda_backend() for --backend cuda (runtime/main.cpp:564-573).
#pragma once

#include <memory>

#include "backend.h"

std::unique_ptr<tinyqwen::IBackend> create_b200_backend();
