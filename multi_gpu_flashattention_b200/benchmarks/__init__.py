"""Benchmark and checking entry points (python -m multi_gpu_flashattention_b200.benchmarks.X).

ring_attention     the reference's ring/attention/bench drivers (one --backend flag)
ring_loop          the reference's ring/loop pure-exchange benchmarks
check_peer         peer-access / NVLink topology report (ring/check_peer.cu)
single_gpu_shapes  single-GPU attention timing over shapes (tests/benchmark_single_gpu_shapes.py)
"""
