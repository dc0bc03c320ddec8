#!/bin/bash
# Regenerates the reference-engine golden fixtures by running the reference
# Stage 2e scheduler itself (compiled unmodified from the reference tree by
# oracle/ref/Makefile into oracle/_ref/ref_run) on one GPU, fed the synthetic
# stream snn_b200.stream(200000, seed=7) as its text corpus:
#   ref_b200_stage2e_seed7_spikes.txt  step, spike count, FNV-1a 64 of the
#                                      spiking neuron indices (int32), 300 steps
#   ref_b200_stage2e_seed7_state.npz   V / w / fire rate of every 11th neuron
#                                      and the alpha / beta sums after 300 steps
# Usage (on a GPU machine, from the repository root, after building):
#   bash tests/golden/make_ref_gpu_pin.sh
set -e
cd "$(dirname "$0")/../.."
out=$(mktemp -d)
python -c "
import sys; sys.path.insert(0,'pure-snn-language_b200')
import snn_b200 as snn
open('$out/corpus.bin','wb').write(snn.stream(200000, seed=7).tobytes())"
oracle/_ref/ref_run --steps 300 --corpus "$out/corpus.bin" --dump "$out/spikes.txt" --state "$out/state.bin"
cp "$out/spikes.txt" tests/golden/ref_b200_stage2e_seed7_spikes.txt
python -c "
import numpy as np
raw = np.fromfile('$out/state.bin', dtype=np.uint8); N = 55000
f = raw[:3*N*4].view(np.float32).reshape(3, N); sa, sb = raw[3*N*4:].view(np.float64)
idx = np.arange(0, N, 11)
np.savez_compressed('tests/golden/ref_b200_stage2e_seed7_state.npz', idx=idx, V=f[0][idx],
                    w=f[1][idx], fr=f[2][idx], alpha_sum=sa, beta_sum=sb)"
