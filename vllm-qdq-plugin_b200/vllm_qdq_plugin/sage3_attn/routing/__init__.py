# SPDX-License-Identifier: Apache-2.0
"""Per-(layer, denoising-step) routing of the Sage3 attention config."""
