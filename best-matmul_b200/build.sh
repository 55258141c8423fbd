#!/usr/bin/env bash
# Build the B200 GEMM library and one benchmark binary per kernel variant,
# then write manifest.tsv (the contract run.sh reads; never guessed from file
# names). Compiles only: no GPU is needed or queried.
#
#   bash build.sh [--suite core|sweep|all] [--output-dir DIR] [--with-validation]
#                 [--nvcc PATH] [--dry-run] [--help]
#
# core : the five tcgen05 variants plus the shape-chosen "auto" build
# sweep: the same variants with strict tile checks off (ragged shapes allowed)
# manifest.tsv keeps the reference's first twelve columns
#   id version cta_m cta_n cta_k pipe gmma_n compute_threads producer_threads
#   inflight epilogue binary
# with sm_100a meanings (cta_m/cta_n = output tile of a CTA pair or CTA,
# gmma_n = N of one tcgen05.mma, compute_threads = epilogue threads,
# producer_threads = 32 (one TMA warp), inflight = TMEM accumulator stages,
# epilogue = 1 (TMEM -> smem -> TMA store)) and appends cta_group,
# mma_per_k, variant and strict.
set -euo pipefail

here="$(cd -- "$(dirname -- "${BASH_SOURCE[0]}")" && pwd -P)"
root="$(cd -- "$here/.." && pwd -P)"
suite=core
output_dir="$here/build/core"
output_set=0
with_validation=0
dry_run=0
nvcc="${CUDACXX:-}"

usage() {
  sed -n '2,20p' "${BASH_SOURCE[0]}" | sed 's/^# \{0,1\}//'
}
fail() { printf 'build.sh: %s\n' "$1" >&2; exit 2; }
need_value() { (( $# >= 2 )) && [[ -n "$2" && "$2" != --* ]] || fail "Missing value for $1"; }

while (( $# )); do
  case "$1" in
    --suite) need_value "$@"; suite="$2"; shift 2 ;;
    --output-dir) need_value "$@"; output_dir="$2"; output_set=1; shift 2 ;;
    --with-validation) with_validation=1; shift ;;
    --nvcc) need_value "$@"; nvcc="$2"; shift 2 ;;
    --dry-run) dry_run=1; shift ;;
    --help|-h) usage; exit 0 ;;
    *) usage >&2; fail "Unknown option: $1" ;;
  esac
done
case "$suite" in core|sweep|all) ;; *) fail "--suite must be core, sweep or all" ;; esac
(( output_set )) || output_dir="$here/build/$suite"
[[ "$output_dir" == /* ]] || output_dir="$PWD/$output_dir"
if [[ -z "$nvcc" ]]; then
  if [[ -x /usr/local/cuda/bin/nvcc ]]; then nvcc=/usr/local/cuda/bin/nvcc; else nvcc=nvcc; fi
fi
for path in "$output_dir" "$nvcc"; do
  [[ "$path" != *$'\t'* && "$path" != *$'\n'* ]] || fail "Paths must not contain tabs or newlines"
done

# id variant cta_group cta_m cta_n pipe mma_n mma_per_k inflight strict
core_variants=(
  'sm100_auto 0 2 256 512 4 256 2 1 1'
  'sm100_2cta_256x512 5 2 256 512 4 256 2 1 1'
  'sm100_2cta_256x256 1 2 256 256 6 256 1 2 1'
  'sm100_1cta_128x256 2 1 128 256 4 256 1 2 1'
  'sm100_1cta_128x128 3 1 128 128 6 128 1 2 1'
  'sm100_2cta_256x128 4 2 256 128 6 128 1 2 1'
)
sweep_variants=(
  'sm100_auto_ragged 0 2 256 512 4 256 2 1 0'
  'sm100_2cta_256x512_ragged 5 2 256 512 4 256 2 1 0'
  'sm100_1cta_128x256_ragged 2 1 128 256 4 256 1 2 0'
)
variants=()
[[ "$suite" == sweep ]] || variants+=("${core_variants[@]}")
[[ "$suite" == core ]] || variants+=("${sweep_variants[@]}")

header=$'id\tversion\tcta_m\tcta_n\tcta_k\tpipe\tgmma_n\tcompute_threads\tproducer_threads\tinflight\tepilogue\tbinary\tcta_group\tmma_per_k\tvariant\tstrict'
lib_dir="$here/lib"
common=(-gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -lineinfo
        "-L$lib_dir" -lbmgemm -Xlinker -rpath -Xlinker "$lib_dir")

commands_for() {  # id variant strict -> sets build_cmd, validate_cmd
  local id="$1" variant="$2" strict="$3"
  local defs=("-DSM100_VARIANT=$variant" "-DSM100_STRICT=$strict")
  build_cmd=("$nvcc" "${common[@]}" "${defs[@]}" "$here/harness/benchmark_host.cu" -o "$output_dir/$id")
  validate_cmd=("$nvcc" "${common[@]}" "${defs[@]}" "$here/harness/full_output_validation.cu"
                -o "$output_dir/$id.validate")
}

print_cmd() { printf '%q ' "$@"; printf '\n'; }

if (( dry_run )); then
  printf '# suite=%s variants=%d with_validation=%s output=%s\n' "$suite" "${#variants[@]}" \
    "$with_validation" "$output_dir"
  print_cmd python3 "$here/build.py" --lib-only
  printf '%s\n' "$header"
  for row in "${variants[@]}"; do
    read -r id variant cg cm cn pipe mn mk infl strict <<< "$row"
    commands_for "$id" "$variant" "$strict"
    print_cmd "${build_cmd[@]}"
    (( with_validation )) && print_cmd "${validate_cmd[@]}"
  done
  exit 0
fi

command -v "$nvcc" >/dev/null 2>&1 || fail "CUDA compiler not found: $nvcc"
mkdir -p -- "$output_dir"
python3 "$here/build.py" --lib-only
[[ -f "$lib_dir/libbmgemm.so" ]] || fail "library build failed"

# manifest is replaced atomically once every build succeeded
tmp="$output_dir/.manifest.tsv.$$"
trap 'rm -f -- "$tmp"' EXIT
printf '%s\n' "$header" > "$tmp"
{
  printf 'build_utc=%s\nsuite=%s\nwith_validation=%s\nnvcc=%s\n' \
    "$(date -u +%Y-%m-%dT%H:%M:%SZ)" "$suite" "$with_validation" "$nvcc"
  "$nvcc" --version 2>/dev/null | tail -1
  git -C "$root" rev-parse HEAD 2>/dev/null || true
} > "$output_dir/build_env.txt"
for row in "${variants[@]}"; do
  read -r id variant cg cm cn pipe mn mk infl strict <<< "$row"
  commands_for "$id" "$variant" "$strict"
  print_cmd "${build_cmd[@]}" >> "$output_dir/commands.sh"
  "${build_cmd[@]}" > "$output_dir/$id.build.log" 2>&1 || { cat "$output_dir/$id.build.log" >&2; fail "build failed: $id"; }
  if (( with_validation )); then
    print_cmd "${validate_cmd[@]}" >> "$output_dir/commands.sh"
    "${validate_cmd[@]}" > "$output_dir/$id.validate.build.log" 2>&1 || { cat "$output_dir/$id.validate.build.log" >&2; fail "validation build failed: $id"; }
    "$output_dir/$id.validate" --mapping-only > "$output_dir/$id.mapping.txt" 2>&1 || fail "mapping check failed: $id"
  fi
  "$output_dir/$id" --help > "$output_dir/$id.help.txt" 2>&1 || fail "--help failed: $id"
  sha256sum "$output_dir/$id" > "$output_dir/$id.sha256.txt" 2>/dev/null || true
  printf '%s\t%s\t%s\t%s\t%s\t%s\t%s\t%s\t%s\t%s\t%s\t%s\t%s\t%s\t%s\t%s\n' \
    "$id" sm100 "$cm" "$cn" 64 "$pipe" "$mn" 256 32 "$infl" 1 "$output_dir/$id" \
    "$cg" "$mk" "$variant" "$strict" >> "$tmp"
done
mv -- "$tmp" "$output_dir/manifest.tsv"
trap - EXIT
printf 'Built %d variants; manifest: %s\n' "${#variants[@]}" "$output_dir/manifest.tsv"
