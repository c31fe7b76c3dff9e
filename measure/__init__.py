"""Measurement drivers of the benchmark configurations beside ``bench.py``.

* ``measure.sweep`` -- config 3: one config-1 layer at 32K-512K tokens, on
  1 GPU or sequence-parallel under torchrun;
* ``measure.batched`` -- config 4: the batched 24-layer small model,
  data-parallel under torchrun;
* ``measure.profile_case`` -- one hot-path layer for profilers;
* ``measure.inputs`` -- the seeded synthetic inputs they share with the tests.
"""
