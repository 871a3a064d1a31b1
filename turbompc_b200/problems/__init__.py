"""Problem definitions and synthetic QP generators."""
