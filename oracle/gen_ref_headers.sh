#!/bin/sh
# Turns the reference's C++23 named-module sources (.ixx) into textual headers so that
# g++ 13 (which cannot build named modules through a module scanner) compiles them as-is.
# The transform is purely mechanical and the output goes to a scratch directory given
# as $2; nothing generated here is committed or shipped.
#   $1 = reference root (the read-only checkout), $2 = output directory
#   $3 = "backend" (optional): the engine's TensorStorage and CUDABackend modules become
#        forwarding headers to this repository's replacements (include/om_tensor_storage.hpp,
#        include/om_cuda_backend.hpp), for a build of the engine on the B200 backend
set -e
REF="$1"; OUT="$2"; MODE="$3"
mkdir -p "$OUT"
for f in "$REF"/src/hal/om.hal.simd.ixx "$REF"/src/hal/om.hal.cpu_backend.ixx \
         "$REF"/src/hal/om.hal.cuda_backend.ixx \
         "$REF"/src/engine/om.engine.tensor_storage.ixx "$REF"/src/engine/om.engine.tensor.ixx \
         "$REF"/src/engine/om.engine.autograd.ixx "$REF"/src/engine/om.engine.tensor_ops.ixx \
         "$REF"/src/engine/om.engine.module.ixx "$REF"/src/engine/om.engine.linear.ixx \
         "$REF"/src/engine/om.engine.activations.ixx "$REF"/src/engine/om.engine.conv.ixx \
         "$REF"/src/engine/om.engine.resnet.ixx "$REF"/src/engine/om.engine.resnet50.ixx \
         "$REF"/src/engine/om.engine.mobilenet.ixx "$REF"/src/engine/om.engine.optimizer.ixx \
         "$REF"/src/engine/om.engine.loss.ixx "$REF"/src/engine/om.engine.serializer.ixx; do
  b=$(basename "$f" .ixx)
  { echo '#pragma once'; \
    sed -e 's/^module;.*$//' -e 's/^export module .*;.*$//' \
        -e 's/^import \(om\.[a-z_.0-9]*\);.*$/#include "\1.hpp"/' \
        -e 's/^export namespace/namespace/' -e 's/^export //' "$f"; } > "$OUT/$b.hpp"
done
if [ "$MODE" = "backend" ]; then
  printf '#pragma once\n#include "om_tensor_storage.hpp"\n' > "$OUT/om.engine.tensor_storage.hpp"
  printf '#pragma once\n#include "om_cuda_backend.hpp"\n' > "$OUT/om.hal.cuda_backend.hpp"
fi
