// matrix.h -- the iq_matrix handle behind the operator-level C ABI.
#pragma once
#include <memory>
#include "api_util.h"
#include "qmv.cuh"

struct iq_matrix {
  int dtype;
  int64_t rows, cols, row_bytes;
  std::shared_ptr<iq::DevBuf> storage;
  const uint8_t* base;
  // Device copy of the last job table this matrix launched, reused while the
  // call's buffers and row count stay the same.
  std::shared_ptr<iq::DevBuf> job_cache = std::make_shared<iq::DevBuf>();
  iq::QmvJob last_job = {};
};

