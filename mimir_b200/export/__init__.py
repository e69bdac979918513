"""Export of trained checkpoints to the Hugging Face Mimir2 format."""
