"""predicitivecoding_b200 — predictive-coding networks and decoder LMs on NVIDIA B200.

Layers: ``models`` (decoder LM, configs), ``engine`` (fused device trainers),
``ops`` (sm_100a kernels), ``parallel`` (data/tensor parallel over NVLink),
``pc`` (predictive-coding engine), ``llm`` (tokenizers, eval, generation, facade),
``io`` (checkpoint formats), ``optim`` (optimizers, schedules), ``utils``.
"""
__version__ = "0.1.0"
