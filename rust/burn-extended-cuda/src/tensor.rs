//! Owned CUDA device buffers holding row-major tensors: the activation type of
//! this crate's `forward` (the reference's Burn `Tensor<B, 3>` on WGPU).
use std::ffi::c_void;
use std::ptr;

use crate::error::{cuda_check, MxMoeError};
use crate::sys::{self, cudart};

/// Element type of activations and biases.
#[derive(Debug, Clone, Copy, PartialEq, Eq)]
pub enum DType {
    F32,
    BF16,
}

impl DType {
    pub fn size(self) -> usize {
        match self {
            DType::F32 => 4,
            DType::BF16 => 2,
        }
    }
    pub fn code(self) -> sys::mxmoe_dtype {
        match self {
            DType::F32 => sys::MXMOE_F32,
            DType::BF16 => sys::MXMOE_BF16,
        }
    }
}

/// A `D`-dimensional row-major tensor in device memory of one CUDA device.
/// `forward` consumes its input by value like the reference's Burn tensors.
#[derive(Debug)]
pub struct DeviceTensor<const D: usize> {
    ptr: *mut c_void,
    shape: [usize; D],
    dtype: DType,
    device: i32,
}

unsafe impl<const D: usize> Send for DeviceTensor<D> {}

impl<const D: usize> DeviceTensor<D> {
    /// Uninitialized device tensor.
    pub fn empty(shape: [usize; D], dtype: DType, device: i32) -> Result<Self, MxMoeError> {
        let bytes = shape.iter().product::<usize>() * dtype.size();
        let mut p: *mut c_void = ptr::null_mut();
        unsafe {
            cuda_check(cudart::cudaSetDevice(device), "cudaSetDevice")?;
            if bytes > 0 {
                cuda_check(cudart::cudaMalloc(&mut p, bytes), "cudaMalloc")?;
            }
        }
        Ok(Self { ptr: p, shape, dtype, device })
    }

    /// Copies host elements (f32 or bf16 bit patterns as `u16`) to a new tensor.
    pub fn from_host<T: Copy>(data: &[T], shape: [usize; D], dtype: DType, device: i32) -> Result<Self, MxMoeError> {
        assert_eq!(std::mem::size_of::<T>(), dtype.size(), "host element size does not match dtype");
        assert_eq!(data.len(), shape.iter().product::<usize>(), "host data does not match shape");
        let t = Self::empty(shape, dtype, device)?;
        if !data.is_empty() {
            unsafe {
                cuda_check(
                    cudart::cudaMemcpy(t.ptr, data.as_ptr() as *const c_void, t.bytes(), cudart::CUDA_MEMCPY_HOST_TO_DEVICE),
                    "cudaMemcpy H2D",
                )?;
            }
        }
        Ok(t)
    }

    /// Copies the tensor to a host vector of `T` (4-byte `f32` or 2-byte bf16 bits).
    pub fn to_host<T: Copy + Default>(&self) -> Result<Vec<T>, MxMoeError> {
        assert_eq!(std::mem::size_of::<T>(), self.dtype.size(), "host element size does not match dtype");
        let mut v = vec![T::default(); self.numel()];
        if !v.is_empty() {
            unsafe {
                cuda_check(cudart::cudaSetDevice(self.device), "cudaSetDevice")?;
                cuda_check(cudart::cudaDeviceSynchronize(), "cudaDeviceSynchronize")?;
                cuda_check(
                    cudart::cudaMemcpy(v.as_mut_ptr() as *mut c_void, self.ptr, self.bytes(), cudart::CUDA_MEMCPY_DEVICE_TO_HOST),
                    "cudaMemcpy D2H",
                )?;
            }
        }
        Ok(v)
    }

    pub fn dims(&self) -> [usize; D] {
        self.shape
    }
    pub fn dtype(&self) -> DType {
        self.dtype
    }
    pub fn device(&self) -> i32 {
        self.device
    }
    pub fn numel(&self) -> usize {
        self.shape.iter().product()
    }
    pub fn bytes(&self) -> usize {
        self.numel() * self.dtype.size()
    }
    pub fn as_ptr(&self) -> *const c_void {
        self.ptr
    }
    pub fn as_mut_ptr(&mut self) -> *mut c_void {
        self.ptr
    }
}

impl<const D: usize> Drop for DeviceTensor<D> {
    fn drop(&mut self) {
        if !self.ptr.is_null() {
            unsafe {
                cudart::cudaSetDevice(self.device);
                cudart::cudaFree(self.ptr);
            }
        }
    }
}
