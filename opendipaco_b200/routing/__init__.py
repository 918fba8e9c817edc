from .base import BagOfTokensFeaturizer, Featurizer, Router
from .discriminative import DiscriminativeRouter
from .featurizers import EmbeddingFeaturizer, HFEncoderFeaturizer, ModelFeaturizer
from .kmeans import KMeansRouter

__all__ = ["Featurizer", "Router", "BagOfTokensFeaturizer", "EmbeddingFeaturizer",
           "ModelFeaturizer", "HFEncoderFeaturizer", "KMeansRouter", "DiscriminativeRouter"]
