"""Estimator registry (``skmetal/estimators/_registry.py:23-51``).

KMeans maps to the CUDA implementation unconditionally; the reference only
registered it when the MLX flash-kmeans backend imported.
"""

from sklearn.cluster import KMeans

GPU_REGISTRY: dict[type, tuple[str, str]] = {
    KMeans: ("skmetal_b200.estimators.cluster", "MetalKMeans"),
}
