// common/types/tensor3d.hpp -- host 3-D array in the reference's layout.
//
// Dimensions from innermost to outermost: columns, rows, sheets; element
// (col, row, sheet) lives at sheet*rows*cols + row*cols + col
// (include/common/types/tensor3d.hpp:107-112 in gpu_algos).  This version has
// no Eigen dependency: the views it hands out (rows, sheets, row-chips) are
// plain strided spans with the few operations the GLM host code needs.
#pragma once

#include <array>
#include <cstddef>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

#include <cuda_fp16.h>

#include "common/random.hpp"

// A strided 1-D view (a row of a Tensor3D, or a column through sheets).
template <typename Number>
class Tensor3DSpan {
   public:
    Tensor3DSpan(Number* data, long size, long stride = 1) : data_(data), size_(size), stride_(stride) {}
    long size() const { return size_; }
    Number& operator[](long i) const { return data_[i * stride_]; }
    Number& operator()(long i) const { return data_[i * stride_]; }
    // Dot product in the element type (the reference's Eigen row.dot(row)).
    template <typename Other>
    std::remove_const_t<Number> dot(const Tensor3DSpan<Other>& other) const {
        if (other.size() != size_) throw std::invalid_argument("dot: size mismatch");
        using R = std::remove_const_t<Number>;
        R s = R(0);
        for (long i = 0; i < size_; ++i) s += (*this)[i] * other[i];
        return s;
    }

   private:
    Number* data_;
    long size_;
    long stride_;
};

template <typename Number>
class Tensor3D {
   public:
    using Row = Tensor3DSpan<Number>;
    using Row_const = Tensor3DSpan<const Number>;

    const long ncols_;
    const long nrows_;
    const long nsheets_;
    std::vector<Number> vector_;

    Tensor3D(const long ncols, const long nrows, const long nsheets, const Number init_value = Number{})
        : ncols_(ncols), nrows_(nrows), nsheets_(nsheets),
          vector_(static_cast<size_t>(ncols) * static_cast<size_t>(nrows) * static_cast<size_t>(nsheets), init_value) {
        if (ncols < 0 || nrows < 0 || nsheets < 0) throw std::invalid_argument("Tensor3D: negative dimension");
    }
    Tensor3D(const Tensor3D& other) = default;
    Tensor3D(Tensor3D&& other) = default;

    long cols() const { return ncols_; }
    long rows() const { return nrows_; }
    long sheets() const { return nsheets_; }
    std::array<long, 3> dims() const { return {ncols_, nrows_, nsheets_}; }
    Number* data() { return vector_.data(); }
    const Number* data() const { return vector_.data(); }

    long row_size() const { return ncols_; }
    long sheet_size() const { return nrows_ * ncols_; }
    long tensor_size() const { return nsheets_ * sheet_size(); }

    std::size_t iat(const long col, const long row, const long sheet) const {
        if (col < 0 || col >= ncols_)
            throw std::invalid_argument("col out of bounds: col=" + std::to_string(col) + " ncols_=" + std::to_string(ncols_));
        if (row < 0 || row >= nrows_)
            throw std::invalid_argument("row out of bounds: row=" + std::to_string(row) + " nrows_=" + std::to_string(nrows_));
        if (sheet < 0 || sheet >= nsheets_)
            throw std::invalid_argument("sheet out of bounds: sheet=" + std::to_string(sheet) + " nsheets_=" + std::to_string(nsheets_));
        return static_cast<std::size_t>(sheet) * sheet_size() + static_cast<std::size_t>(row) * row_size() + col;
    }
    Number& operator()(const long col, const long row, const long sheet) {
        return vector_[static_cast<std::size_t>(sheet) * sheet_size() + static_cast<std::size_t>(row) * row_size() + col];
    }
    const Number& operator()(const long col, const long row, const long sheet) const {
        return vector_[static_cast<std::size_t>(sheet) * sheet_size() + static_cast<std::size_t>(row) * row_size() + col];
    }
    Number& at(const long col, const long row, const long sheet) { return vector_[iat(col, row, sheet)]; }
    const Number& at(const long col, const long row, const long sheet) const { return vector_[iat(col, row, sheet)]; }

    // The contiguous row (row, sheet): ncols elements.
    Row row_at(const long row, const long sheet) { return Row(&vector_[iat(0, row, sheet)], ncols_); }
    Row_const row_at(const long row, const long sheet) const { return Row_const(&vector_[iat(0, row, sheet)], ncols_); }

    void randomize(const long seed) { randomize_container(vector_, seed); }

    template <typename OSTREAM>
    void print(OSTREAM& os) const {
        using Printable = std::conditional_t<std::is_floating_point_v<Number>, Number,
                                             std::conditional_t<std::is_same_v<Number, __half>, float, long long>>;
        for (long sheet = 0; sheet < nsheets_; ++sheet) {
            for (long row = 0; row < nrows_; ++row) {
                os << "(" << sheet << "," << row << "): [ ";
                for (long col = 0; col < ncols_; ++col) {
                    if constexpr (std::is_same_v<Number, __half>) os << __half2float((*this)(col, row, sheet)) << " ";
                    else os << static_cast<Printable>((*this)(col, row, sheet)) << " ";
                }
                os << "]\n";
            }
        }
    }
};
