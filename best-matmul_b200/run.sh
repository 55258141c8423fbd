#!/usr/bin/env bash
# Run the binaries listed in a build's manifest.tsv (see build.sh).
#
#   bash run.sh --mode env|check|validate|bench|ncu|all [options]
#
# Modes
#   env       environment snapshot (no kernels)
#   check     each binary on 2x2 tiles, K tiles {1, 2, S, S+1, 2S+1}, 16+48
#             sampled entries against the FP64 reference (input mode 3)
#   validate  each <binary>.validate: every C element of small problems, bit exact
#   bench     shapes x layouts x repeats, rotated variant order; runs.csv and
#             summary.csv (median over processes of the per-process p50)
#   ncu       one GEMM launch per variant/layout under Nsight Compute with
#             --clock-control none (clocks are never locked)
#   all       env + validate + bench + ncu
# nsys (not installed in this image), sanitize (closed on this pool) and
# disasm (reading compiled code is not done in this project) are not offered.
#
# Options
#   --build-dir DIR       directory with manifest.tsv (default build/core)
#   --output-dir DIR      new result directory; must not exist
#   --gpu ID              CUDA device index or UUID for CUDA_VISIBLE_DEVICES (default 0)
#   --variants CSV        manifest ids (default all)
#   --layouts CSV         NT, TN or NT,TN (default both)
#   --shapes CSV          MxNxK list for bench (default 4096x4096x4096,8192x8192x8192)
#   --profile-shape MxNxK ncu problem (default 4096x4096x4096)
#   --repeats N           processes per (variant, shape, layout), >= 2 (default 3)
#   --per-batch N         launches per timed batch (default 20)
#   --min-warmup N        minimum warm-up launches (default 300)
#   --batches N           timed batches, >= 2 (default 100)
#   --baseline ID         summary reference id (default sm100_auto)
#   --ncu PATH            Nsight Compute (default $NCU or ncu)
#   --ncu-set focused|full   sections (default focused)
#   --launch-skip N       GEMM launches skipped before the profiled one (default 50)
#   --timeout SECONDS     per command, 0 = none (default 1800)
#   --dry-run             print commands only
#   --help
set -euo pipefail

here="$(cd -- "$(dirname -- "${BASH_SOURCE[0]}")" && pwd -P)"
mode=bench
build_dir="$here/build/core"
output_dir=""
gpu=0
variants=all
layouts=NT,TN
shapes=4096x4096x4096,8192x8192x8192
profile_shape=4096x4096x4096
repeats=3
per_batch=20
min_warmup=300
batches=100
baseline=sm100_auto
ncu_bin="${NCU:-ncu}"
ncu_set=focused
launch_skip=50
timeout_sec=1800
dry_run=0
nvidia_smi="${NVIDIA_SMI:-nvidia-smi}"

usage() { sed -n '2,35p' "${BASH_SOURCE[0]}" | sed 's/^# \{0,1\}//'; }
die() { printf 'run.sh: %s\n' "$*" >&2; exit 1; }
need_value() { (( $# >= 2 )) && [[ -n "$2" && "$2" != --* ]] || die "Missing value for $1"; }
positive() { [[ "$2" =~ ^[1-9][0-9]*$ ]] || die "$1 must be a positive integer"; }

while (( $# )); do
  case "$1" in
    --help|-h) usage; exit 0 ;;
    --dry-run) dry_run=1; shift ;;
    --mode) need_value "$@"; mode="$2"; shift 2 ;;
    --build-dir) need_value "$@"; build_dir="$2"; shift 2 ;;
    --output-dir) need_value "$@"; output_dir="$2"; shift 2 ;;
    --gpu) need_value "$@"; gpu="$2"; shift 2 ;;
    --variants) need_value "$@"; variants="$2"; shift 2 ;;
    --layouts) need_value "$@"; layouts="$2"; shift 2 ;;
    --shapes) need_value "$@"; shapes="$2"; shift 2 ;;
    --profile-shape) need_value "$@"; profile_shape="$2"; shift 2 ;;
    --repeats) need_value "$@"; repeats="$2"; shift 2 ;;
    --per-batch) need_value "$@"; per_batch="$2"; shift 2 ;;
    --min-warmup) need_value "$@"; min_warmup="$2"; shift 2 ;;
    --batches) need_value "$@"; batches="$2"; shift 2 ;;
    --baseline) need_value "$@"; baseline="$2"; shift 2 ;;
    --ncu) need_value "$@"; ncu_bin="$2"; shift 2 ;;
    --ncu-set) need_value "$@"; ncu_set="$2"; shift 2 ;;
    --launch-skip) need_value "$@"; launch_skip="$2"; shift 2 ;;
    --timeout) need_value "$@"; timeout_sec="$2"; shift 2 ;;
    *) usage >&2; die "Unknown option: $1" ;;
  esac
done

case "$mode" in
  env|check|validate|bench|ncu|all) ;;
  nsys) die "nsys mode: Nsight Systems is not installed in this image" ;;
  sanitize) die "sanitize mode: compute-sanitizer is closed on this pool" ;;
  disasm) die "disasm mode is not provided: this project does not read compiled code" ;;
  *) die "Unknown mode: $mode" ;;
esac
for v in repeats per_batch min_warmup batches launch_skip; do positive "--${v//_/-}" "${!v}"; done
(( repeats >= 2 )) || die "--repeats must be at least 2"
(( batches >= 2 )) || die "--batches must be at least 2"
[[ "$timeout_sec" =~ ^[0-9]+$ ]] || die "--timeout must be a non-negative integer"
case "$ncu_set" in focused|full) ;; *) die "--ncu-set must be focused or full" ;; esac
[[ "$build_dir" == /* ]] || build_dir="$PWD/$build_dir"
IFS=, read -r -a layout_list <<< "$layouts"
IFS=, read -r -a shape_list <<< "$shapes"
for l in "${layout_list[@]}"; do [[ "$l" == NT || "$l" == TN ]] || die "Unsupported layout: $l"; done

# ---------------------------------------------------------------- manifest
declare -a ids=()
declare -A cta_m cta_n cta_k pipes binary strictness
if [[ "$mode" != env ]]; then
  [[ -f "$build_dir/manifest.tsv" ]] || die "No manifest.tsv in $build_dir; run build.sh first"
  expected=$'id\tversion\tcta_m\tcta_n\tcta_k\tpipe\tgmma_n\tcompute_threads\tproducer_threads\tinflight\tepilogue\tbinary\tcta_group\tmma_per_k\tvariant\tstrict'
  IFS= read -r header < "$build_dir/manifest.tsv"
  [[ "$header" == "$expected" ]] || die "manifest.tsv header does not match this runner; rebuild"
  while IFS=$'\t' read -r id ver cm cn ck pp gn ct pt infl ep bin cg mk var strict; do
    [[ "$id" =~ ^[A-Za-z0-9_]+$ && -z "${binary[$id]+x}" ]] || die "Bad or duplicate manifest id: $id"
    [[ "$ver" == sm100 ]] || die "Unsupported manifest version for $id: $ver"
    for value in "$cm" "$cn" "$ck" "$pp" "$gn" "$ct" "$pt" "$infl"; do
      [[ "$value" =~ ^[1-9][0-9]{0,4}$ ]] || die "Bad manifest number for $id"
    done
    [[ "$ep" =~ ^[01]$ && "$cg" =~ ^[12]$ && "$mk" =~ ^[12]$ && "$var" =~ ^[0-5]$ && "$strict" =~ ^[01]$ ]] ||
      die "Bad manifest configuration for $id"
    [[ "$bin" == /* ]] || die "Binary path must be absolute for $id"
    cta_m[$id]="$cm"; cta_n[$id]="$cn"; cta_k[$id]="$ck"; pipes[$id]="$pp"; binary[$id]="$bin"
    strictness[$id]="$strict"
    ids+=("$id")
  done < <(tail -n +2 "$build_dir/manifest.tsv")
  (( ${#ids[@]} )) || die "manifest.tsv lists no variants"
  if [[ "$variants" != all ]]; then
    IFS=, read -r -a wanted <<< "$variants"
    declare -A seen=()
    for id in "${wanted[@]}"; do
      [[ -n "${binary[$id]+x}" ]] || die "Not in manifest: $id"
      [[ -z "${seen[$id]+x}" ]] || die "Duplicate id: $id"
      seen[$id]=1
    done
    ids=("${wanted[@]}")
  fi
fi

parse_shape() {
  [[ "$1" =~ ^([1-9][0-9]{0,8})x([1-9][0-9]{0,8})x([1-9][0-9]{0,8})$ ]] || die "Shape must be MxNxK: $1"
  m="${BASH_REMATCH[1]}"; n="${BASH_REMATCH[2]}"; k="${BASH_REMATCH[3]}"
  (( m * n <= 2147483647 && m * k <= 2147483647 && n * k <= 2147483647 )) || die "Too many elements: $1"
  local id
  for id in "${ids[@]}"; do
    if (( strictness[$id] )); then
      (( m % cta_m[$id] == 0 && n % cta_n[$id] == 0 && k % cta_k[$id] == 0 )) ||
        die "$1 is not a multiple of $id's tile (${cta_m[$id]}x${cta_n[$id]}x${cta_k[$id]})"
    fi
  done
}
if [[ "$mode" == bench || "$mode" == all ]]; then for s in "${shape_list[@]}"; do parse_shape "$s"; done; fi
if [[ "$mode" == ncu || "$mode" == all ]]; then parse_shape "$profile_shape"; fi

[[ -n "$output_dir" ]] || output_dir="$here/results/$(date +%Y%m%d_%H%M%S)_${mode}_$$"
[[ "$output_dir" == /* ]] || output_dir="$PWD/$output_dir"

# ---------------------------------------------------------------- device gate
# Kernels need compute capability 10.0 (B200). The query goes through
# nvidia-smi so the gate works before any CUDA context exists.
device_gate() {
  local cap name
  cap="$("$nvidia_smi" -i "$gpu" --query-gpu=compute_cap --format=csv,noheader 2>/dev/null | head -1 | tr -d ' ')" ||
    die "nvidia-smi could not query GPU $gpu"
  name="$("$nvidia_smi" -i "$gpu" --query-gpu=name --format=csv,noheader 2>/dev/null | head -1)"
  [[ "$cap" == 10.0 ]] || die "GPU $gpu ($name) has compute capability ${cap:-unknown}; these kernels need 10.0 (B200)"
}

record_command() { printf '%q ' "$@" >> "$output_dir/commands.sh"; printf '\n' >> "$output_dir/commands.sh"; }

run_logged() {  # log cmd... : run under timeout, keep output, fail loudly
  local log="$1"; shift
  local -a cmd=("$@")
  (( timeout_sec == 0 )) || cmd=(timeout --kill-after=30s "${timeout_sec}s" "${cmd[@]}")
  if (( dry_run )); then printf '%q ' "${cmd[@]}"; printf '\n'; return 0; fi
  record_command "${cmd[@]}"
  printf '%s\tstart\t%s\n' "$(date -u +%Y-%m-%dT%H:%M:%S.%NZ)" "$log" >> "$output_dir/timeline.tsv"
  local code=0
  CUDA_VISIBLE_DEVICES="$gpu" "${cmd[@]}" > "$output_dir/$log" 2>&1 || code=$?
  printf '%s\tend\t%s\t%s\n' "$(date -u +%Y-%m-%dT%H:%M:%S.%NZ)" "$log" "$code" >> "$output_dir/timeline.tsv"
  if (( code != 0 )); then
    tail -n 30 -- "$output_dir/$log" >&2
    die "command failed (exit $code); see $output_dir/$log"
  fi
}

collect_environment() {
  (( dry_run )) && return 0
  { date -u; uname -a; } > "$output_dir/env_host.txt" 2>&1 || true
  "$nvidia_smi" -q > "$output_dir/env_nvidia_smi.txt" 2>&1 || true
  "$nvidia_smi" --query-gpu=index,name,uuid,compute_cap,clocks.sm,clocks.max.sm,power.limit \
    --format=csv > "$output_dir/env_gpus.csv" 2>&1 || true
  nvcc --version > "$output_dir/env_nvcc.txt" 2>&1 || true
  "$ncu_bin" --version > "$output_dir/env_ncu.txt" 2>&1 || true
  if [[ -f "$build_dir/manifest.tsv" ]]; then cp -- "$build_dir/manifest.tsv" "$output_dir/manifest.tsv"; fi
}

run_check() {
  local id layout tiles
  for id in "${ids[@]}"; do
    for layout in "${layout_list[@]}"; do
      declare -A done_tiles=()
      for tiles in 1 2 "${pipes[$id]}" "$((pipes[$id] + 1))" "$((2 * pipes[$id] + 1))"; do
        [[ -z "${done_tiles[$tiles]+x}" ]] || continue
        done_tiles[$tiles]=1
        run_logged "check_${id}_${layout}_k${tiles}.log" "${binary[$id]}" \
          "$((2 * cta_m[$id]))" "$((2 * cta_n[$id]))" "$((tiles * cta_k[$id]))" \
          "${layout:0:1}" "${layout:1:1}" 3 event 1 1 2
      done
      unset done_tiles
    done
  done
}

write_status() {  # id code status start end
  local f="$output_dir/validate_$1.status.tsv"
  { printf 'id\texit_code\tstatus\tstart_utc\tend_utc\tlog\tvalidate_binary\n'
    printf '%s\t%s\t%s\t%s\t%s\t%s\t%s\n' "$1" "$2" "$3" "$4" "$5" "validate_$1.log" "${binary[$1]}.validate"
  } > "$f.tmp" && mv -- "$f.tmp" "$f"
}

run_validate() {
  local id start end code status
  for id in "${ids[@]}"; do
    [[ -x "${binary[$id]}.validate" ]] || die "Missing ${binary[$id]}.validate; build with --with-validation"
    if (( dry_run )); then printf '%q\n' "${binary[$id]}.validate"; continue; fi
    start="$(date -u +%Y-%m-%dT%H:%M:%S.%NZ)"
    write_status "$id" "" RUNNING "$start" ""
    code=0
    local -a cmd=("${binary[$id]}.validate")
    (( timeout_sec == 0 )) || cmd=(timeout --kill-after=30s "${timeout_sec}s" "${cmd[@]}")
    record_command "${cmd[@]}"
    CUDA_VISIBLE_DEVICES="$gpu" "${cmd[@]}" > "$output_dir/validate_$id.log" 2>&1 || code=$?
    end="$(date -u +%Y-%m-%dT%H:%M:%S.%NZ)"
    case "$code" in 0) status=PASS ;; 124) status=TIMEOUT ;; 130|143) status=INTERRUPTED ;; *) status=FAIL ;; esac
    write_status "$id" "$code" "$status" "$start" "$end"
    (( code == 0 )) || { tail -n 30 "$output_dir/validate_$id.log" >&2; die "validation $status for $id"; }
  done
}

run_bench() {
  local shape layout rep j id log
  (( dry_run )) || printf 'id\tshape\tlayout\trepeat\tlog\n' > "$output_dir/bench_index.tsv"
  for shape in "${shape_list[@]}"; do
    parse_shape "$shape"
    for layout in "${layout_list[@]}"; do
      for ((rep = 1; rep <= repeats; ++rep)); do
        # rotate the order each repeat so no variant always runs first (hot/cold GPU)
        for ((j = 0; j < ${#ids[@]}; ++j)); do
          id="${ids[$(((j + rep - 1) % ${#ids[@]}))]}"
          log="bench_${id}_${shape}_${layout}_r${rep}.log"
          run_logged "$log" "${binary[$id]}" "$m" "$n" "$k" "${layout:0:1}" "${layout:1:1}" \
            4 event "$per_batch" "$min_warmup" "$batches"
          (( dry_run )) || printf '%s\t%s\t%s\t%s\t%s\n' "$id" "$shape" "$layout" "$rep" "$log" >> "$output_dir/bench_index.tsv"
        done
      done
    done
  done
  (( dry_run )) && return 0
  python3 "$here/harness/summarize.py" "$output_dir" "$baseline"
}

run_ncu() {
  parse_shape "$profile_shape"
  local -a opts=(--kernel-name regex:bm_gemm_sm100 --launch-skip "$launch_skip" --launch-count 1
                 --clock-control none --replay-mode kernel --cache-control all)
  if [[ "$ncu_set" == full ]]; then opts+=(--set full); else
    for s in LaunchStats Occupancy SpeedOfLight ComputeWorkloadAnalysis MemoryWorkloadAnalysis \
             SchedulerStats WarpStateStats; do opts+=(--section "$s"); done
  fi
  local id layout stem
  for id in "${ids[@]}"; do
    for layout in "${layout_list[@]}"; do
      stem="ncu_${id}_${profile_shape}_${layout}"
      # the same command must first exit 0 without the profiler
      run_logged "$stem.plain.log" "${binary[$id]}" "$m" "$n" "$k" "${layout:0:1}" "${layout:1:1}" \
        4 event 1 "$((launch_skip + 100))" 2
      run_logged "$stem.log" "$ncu_bin" "${opts[@]}" --export "$output_dir/$stem" \
        "${binary[$id]}" "$m" "$n" "$k" "${layout:0:1}" "${layout:1:1}" 4 event 1 "$((launch_skip + 100))" 2
      run_logged "$stem.raw.csv" "$ncu_bin" --import "$output_dir/$stem.ncu-rep" --page raw --csv
    done
  done
}

if (( ! dry_run )); then
  [[ ! -e "$output_dir" ]] || die "Output directory exists: $output_dir (use a new one)"
  mkdir -p -- "$output_dir"
  printf 'utc\tevent\tlog\texit\n' > "$output_dir/timeline.tsv"
  [[ "$mode" == env ]] || device_gate
fi
collect_environment
case "$mode" in
  env) ;;
  check) run_check ;;
  validate) run_validate ;;
  bench) run_bench ;;
  ncu) run_ncu ;;
  all) run_validate; run_bench; run_ncu ;;
esac
(( dry_run )) || printf 'Results in %s\n' "$output_dir"
