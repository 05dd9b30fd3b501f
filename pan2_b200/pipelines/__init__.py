"""Generation pipelines."""
from .video import PanVideoPipeline, PackedDiTRunner, build_inference_model, latent_grid, load_transformer_weights  # noqa: F401
