"""Sampling: Euler scheduler, timestep schedules, guidance plans and prompt inputs."""
