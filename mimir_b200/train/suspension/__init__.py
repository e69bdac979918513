"""Suspendable training: file protocol, in-loop hook, cuda-checkpoint controller, launcher, supervisor."""
