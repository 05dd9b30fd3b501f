from .training import TrainingConfig, build_arg_parser, parse_training_config, load_yaml_defaults  # noqa: F401
