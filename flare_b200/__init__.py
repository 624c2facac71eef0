"""flare_b200: a B200-native (sm_100a) recommendation-training framework.

Entry points: ``flare_b200.training.trainer.DLRMTrainer`` / ``DCNTrainer`` (fused
GPU models), ``flare_b200.training.engine.TrainEngine`` (generic autograd models,
ZeRO 0-3), ``flare_b200.sparse.collection.ShardedEmbeddingBagCollection`` (fused
sharded embeddings), ``flare_b200.sparse.reference.CpuEmbeddingBagCollection``
(CPU configuration), ``flare_b200.cli`` (train / eval) and ``bench.py``.  The
native extension (``flare_b200._C``) is built in-tree by
``python setup.py build_ext --inplace`` and loaded lazily on first use.
"""

__version__ = "0.1.0"
