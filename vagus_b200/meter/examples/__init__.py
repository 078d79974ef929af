"""Worked uses of the meter and diagnostic probes (``python -m
vagus_b200.meter.examples.<name> --help``):

benchmarks (CUDA-event timing through ``meter.compare``)
  bench_attention          our flash attention vs torch SDPA vs materialised scores
  bench_ce                 fused linear cross-entropy vs materialised logits (time, memory)
  bench_linear_attention   the chunked delta-rule family on the kernels vs the torch chunk oracle
  bench_rope               fused qk-norm + RoPE vs plain torch
  bench_dist               all-gather / reduce-scatter bus bandwidth: NVLink kernels vs NCCL (torchrun)
  profile_step             one model's training step under torch.profiler, device time by kernel family

probes on trained checkpoints
  saturation_curve         per-position delta-rule residual |v - S^T k| / |v|: where the state stops learning
  write_selectivity        is the write strength beta selective with respect to that residual
  probe_attention_health   softmax attention sharpness per head: logit ceiling (qk-norm), max cosine, entropy

Parity: reference ``infra/meter/examples/`` (the same questions, answered
with this framework's APIs).
"""
