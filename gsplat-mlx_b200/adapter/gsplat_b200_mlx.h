// MLX-side adapter of gsplat_b200: the `eval_gpu` bodies of the reference's
// eleven gsplat_core Primitives, written over the C ABI of gsplat_b200.h.
//
// The reference defines each `eval_gpu` twice, under `#ifdef _METAL_` (the
// Metal dispatch) and `#else` (a `throw`), e.g. gsplat_rasterize.cpp:571-724
// and :725-738.  A build for CUDA compiles gsplat_b200_eval_gpu.cpp beside
// the reference's sources and drops their `#else` definitions (guard them
// with `#if !defined(GSPLAT_B200)`); everything else of the reference -- the
// front-ends, `eval_cpu`, `vjp`, the nanobind module -- is unchanged.
//
// Every body keeps the reference's contract: outputs allocated with
// `mx::allocator::malloc`, every element written (culled / masked entries as
// exact zeros), the kernels enqueued on the Primitive's stream, shape or
// argument errors thrown as std::runtime_error with the library's message.
#pragma once

#include <cstdint>
#include <vector>

#include "mlx/array.h"
#include "mlx/primitives.h"

namespace gsplat_b200_mlx {

namespace mx = mlx::core;

// Returns the cudaStream_t (as void*) on which MLX runs `stream`, or
// nullptr when none is known.  MLX's CUDA backend keeps one CUDA stream per
// mx::Stream; the host application installs a resolver that looks it up.
using StreamResolver = void* (*)(const mx::Stream& stream);

// Installs the resolver (nullptr: none).  Without a resolver the bodies run
// synchronously: they wait for the device before their launches (so that
// inputs written on any stream are complete) and for the legacy stream after
// them, which is correct whatever streams MLX uses, and slower.
void set_stream_resolver(StreamResolver resolver);

// Stable ascending sort of (isect_ids, flatten_ids) by key -- the result of
// the reference's `mx::argsort` + two `mx::take` in
// gsplat_intersect_tile_sort (gsplat_intersect.cpp:266-286) -- as ONE
// Primitive: on the GPU the radix sort of gs_isect_sort, on the CPU a
// std::stable_sort.  `key_bits` = the reference's image bits + tile bits +
// 32 (only those low key bits may be non-zero).  Returns {sorted_isect_ids,
// sorted_flatten_ids}.  A drop-in for the body of
// gsplat_intersect_tile_sort.
std::vector<mx::array> intersect_tile_sort(const mx::array& isect_ids,
                                           const mx::array& flatten_ids,
                                           int key_bits, mx::StreamOrDevice s = {});

class IntersectSort : public mx::Primitive {
 public:
  IntersectSort(mx::Stream stream, int key_bits)
      : mx::Primitive(stream), key_bits_(key_bits) {}

  void eval_cpu(const std::vector<mx::array>& inputs,
                std::vector<mx::array>& outputs) override;
  void eval_gpu(const std::vector<mx::array>& inputs,
                std::vector<mx::array>& outputs) override;
  std::vector<mx::array> jvp(const std::vector<mx::array>& primals,
                             const std::vector<mx::array>& tangents,
                             const std::vector<int>& argnums) override;
  std::vector<mx::array> vjp(const std::vector<mx::array>& primals,
                             const std::vector<mx::array>& cotangents,
                             const std::vector<int>& argnums,
                             const std::vector<mx::array>& outputs) override;
  std::pair<std::vector<mx::array>, std::vector<int>> vmap(
      const std::vector<mx::array>& inputs,
      const std::vector<int>& axes) override;
  const char* name() const override { return "GSPlatB200IntersectSort"; }
  bool is_equivalent(const mx::Primitive& other) const override;

 private:
  int key_bits_;
};

}  // namespace gsplat_b200_mlx
