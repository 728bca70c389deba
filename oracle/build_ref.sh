#!/usr/bin/env bash
# Builds oracle/_ref/libref_moe.so (MoE kernels) and oracle/_ref/libref_attn.so (decode attention:
# Q8_0 QKV projection + RMSNorm, partial RoPE, split-K GQA decode, Q8_0 matvec) from the
# reference's own CUDA sources, compiled where they lie in the reference tree (nothing is copied
# into this repository).  Test infrastructure only: the golden-vector scripts load them to record
# the reference kernels' outputs.
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${MINIMAX_RS_REFERENCE:-/root/reference}"
SRC="$REF/vendor/candle-kernels/src"
OUT="$HERE/_ref"
LIB="$OUT/libref_moe.so"
LIB_ATTN="$OUT/libref_attn.so"
[ -d "$SRC" ] || { echo "reference tree not found at $REF: skipping"; exit 0; }
mkdir -p "$OUT"
DEPS=("$HERE/build_ref.sh" "$HERE/ref_wrap_dequant.cu" "$HERE/ref_wrap_moe.cu" "$SRC/quantized.cu" "$SRC/moe/moe_gguf.cu" \
      "$SRC/moe/gguf.cuh" "$SRC/moe/moe_sort.cu" "$SRC/mmq_gguf/mmq_moe.cu" "$SRC/mmq_gguf/mmq_quantize.cu" \
      "$SRC/mmq_gguf/mmq_instance_q4_k.cu" "$SRC/mmq_gguf/mmq_instance_q5_k.cu" "$SRC/mmq_gguf/mmq_gguf.cuh")
NVCC="${NVCC:-nvcc}"
FLAGS=(-gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 --expt-relaxed-constexpr -Xcompiler -fPIC)
compile() { "$NVCC" "${FLAGS[@]}" "$@"; }
DEPS_ATTN=("$HERE/build_ref.sh" "$SRC/mmvq_gguf.cu" "$SRC/decode_attention.cu" "$SRC/mmq_gguf/mmq_mma.cuh")
stale=1
if [ -f "$LIB_ATTN" ]; then
  stale=0
  for d in "${DEPS_ATTN[@]}"; do [ "$d" -nt "$LIB_ATTN" ] && stale=1; done
fi
if [ $stale -eq 1 ]; then
  mkdir -p "$OUT/attn"
  compile -I"$SRC" -c "$SRC/mmvq_gguf.cu" -o "$OUT/attn/mmvq_gguf.o" &
  compile -I"$SRC" -c "$SRC/decode_attention.cu" -o "$OUT/attn/decode_attention.o" &
  wait
  "$NVCC" -gencode arch=compute_100a,code=sm_100a -shared -cudart static -o "$LIB_ATTN" "$OUT"/attn/*.o
  echo "built $LIB_ATTN"
fi
if [ -f "$LIB" ]; then
  stale=0
  for d in "${DEPS[@]}"; do [ "$d" -nt "$LIB" ] && stale=1; done
  [ $stale -eq 0 ] && exit 0
fi
compile -I"$SRC" -c "$HERE/ref_wrap_dequant.cu" -o "$OUT/ref_dequant.o" &
compile -I"$SRC/moe" -c "$HERE/ref_wrap_moe.cu" -o "$OUT/ref_moe.o" &
compile -c "$SRC/moe/moe_sort.cu" -o "$OUT/moe_sort.o" &
compile -c "$SRC/mmq_gguf/mmq_moe.cu" -o "$OUT/mmq_moe.o" &
compile -c "$SRC/mmq_gguf/mmq_quantize.cu" -o "$OUT/mmq_quantize.o" &
compile -c "$SRC/mmq_gguf/mmq_instance_q4_k.cu" -o "$OUT/mmq_q4k.o" &
compile -c "$SRC/mmq_gguf/mmq_instance_q5_k.cu" -o "$OUT/mmq_q5k.o" &
wait
"$NVCC" -gencode arch=compute_100a,code=sm_100a -shared -cudart static -o "$LIB" "$OUT"/*.o
echo "built $LIB"
