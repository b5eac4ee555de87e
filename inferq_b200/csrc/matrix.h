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
  // TMA tensor maps over the storage (quantized dtypes): unit box, tail box.
  // Leading-row views share their parent's (rows past the view are read,
  // never stored).
  std::shared_ptr<iq::DevBuf> maps = std::make_shared<iq::DevBuf>();
  const void* tmap() const { return maps->p; }
  const void* tmap_tail() const { return maps->p ? static_cast<const uint8_t*>(maps->p) + 128 : nullptr; }
  // Device copy of the last job table this matrix launched, reused while the
  // call's buffers and row count stay the same.
  std::shared_ptr<iq::DevBuf> job_cache = std::make_shared<iq::DevBuf>();
  iq::QmvJob last_job = {};
};

