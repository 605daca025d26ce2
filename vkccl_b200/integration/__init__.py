# SPDX-License-Identifier: Apache-2.0
"""Integrations with serving frameworks (vLLM)."""
