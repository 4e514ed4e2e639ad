//! Model glue for the MoE blocks.
pub mod gpt_oss;
