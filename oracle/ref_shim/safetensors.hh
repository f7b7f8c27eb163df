// Minimal stand-in for the un-vendored safetensors-cpp header. The reference's
// util/tensor.h only needs the dtype enumeration to compile; nothing here is
// called on the KV-store or index paths.
#pragma once
namespace safetensors {
enum class dtype {
  kBOOL,
  kUINT8,
  kINT8,
  kINT16,
  kUINT16,
  kFLOAT16,
  kBFLOAT16,
  kINT32,
  kUINT32,
  kFLOAT32,
  kFLOAT64,
  kINT64,
  kUINT64,
};
}  // namespace safetensors
